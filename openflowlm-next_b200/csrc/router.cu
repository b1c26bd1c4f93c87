// Router: the logits GEMM and the per-token softmax / top-k. Below the prefill sizes the logits come from
// a split-K kernel (bf16 x bf16 -> f32 on the warp-level tensor cores; the decode sizes are bound by
// reading the router weights, so the K split spreads that read over the SMs); from kRouterTcMinT tokens
// from the tcgen05 kernel of router_tc.cu (routers of more than 496 experts: the logits kernel unsplit).
//
// Follows host::router_block (src/open_qwen36/block_host.cpp:766-803): float logits, max
// subtraction, float exp with a double denominator, p = e * float(1/denom), top-k by probability
// (strictly greater wins, so the lowest index wins a tie), weights renormalised by a double sum.
// The shared-expert gate (core.cpp:4370-4373) rides along as router row E.
#include "common.cuh"
#include "kernels.cuh"

namespace fm {

// xb[t][h] = bf16(xm[t][h]) for f32 input (the rounding the reference applies at the device
// boundary, core.cpp:5204).
__global__ void to_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ xb, long long n4) {
    pdl_wait();
    pdl_launch_dependents();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        uint2 o;
        o.x = pack_bf16x2(v.x, v.y);
        o.y = pack_bf16x2(v.z, v.w);
        reinterpret_cast<uint2*>(xb)[i] = o;
    }
}

__device__ __forceinline__ void mma_bf16_16816(float* c, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Partial logits: part[z][M][N] = A[M, kz] . B[N, kz]^T over the z-th K chunk (kz = K / gridDim.z),
// bf16 in, f32 out. 64x64 CTA tile, 4 warps of 32x32, K step 32 with the next step's operands fetched
// into registers while the current one is multiplied. The top-k kernel sums the chunks in order.
constexpr int RG_BM = 64, RG_BN = 64, RG_BK = 32, RG_LD = RG_BK + 8;
constexpr int kMaxKSplit = 16;

__global__ void __launch_bounds__(128) router_logits_kernel(const uint16_t* __restrict__ A, const uint16_t* __restrict__ B,
                                                            float* __restrict__ part, int M, int N, int K) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ __align__(16) uint16_t sa[2][RG_BM][RG_LD];
    __shared__ __align__(16) uint16_t sb[2][RG_BN][RG_LD];
    const int m0 = blockIdx.y * RG_BM, n0 = blockIdx.x * RG_BN;
    const int kc = K / gridDim.z, kbeg = blockIdx.z * kc;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
    const int g = lane >> 2, c = lane & 3;
    float acc[2][4][4] = {};
    uint4 ra[2], rb[2];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = threadIdx.x + j * 128, r = i >> 2, q = i & 3;
            ra[j] = m0 + r < M ? *reinterpret_cast<const uint4*>(A + (size_t)(m0 + r) * K + k0 + q * 8) : make_uint4(0, 0, 0, 0);
            rb[j] = n0 + r < N ? *reinterpret_cast<const uint4*>(B + (size_t)(n0 + r) * K + k0 + q * 8) : make_uint4(0, 0, 0, 0);
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = threadIdx.x + j * 128, r = i >> 2, q = i & 3;
            *reinterpret_cast<uint4*>(&sa[buf][r][q * 8]) = ra[j];
            *reinterpret_cast<uint4*>(&sb[buf][r][q * 8]) = rb[j];
        }
    };
    fetch(kbeg);
    stash(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = kbeg; k0 < kbeg + kc; k0 += RG_BK) {
        const bool more = k0 + RG_BK < kbeg + kc;
        if (more) fetch(k0 + RG_BK);
#pragma unroll
        for (int kk = 0; kk < RG_BK; kk += 16) {
            uint32_t af[2][4], bf[4][2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int r = wm + i * 16 + g;
                af[i][0] = *reinterpret_cast<const uint32_t*>(&sa[buf][r][kk + 2 * c]);
                af[i][1] = *reinterpret_cast<const uint32_t*>(&sa[buf][r + 8][kk + 2 * c]);
                af[i][2] = *reinterpret_cast<const uint32_t*>(&sa[buf][r][kk + 2 * c + 8]);
                af[i][3] = *reinterpret_cast<const uint32_t*>(&sa[buf][r + 8][kk + 2 * c + 8]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = wn + j * 8 + g;
                bf[j][0] = *reinterpret_cast<const uint32_t*>(&sb[buf][n][kk + 2 * c]);
                bf[j][1] = *reinterpret_cast<const uint32_t*>(&sb[buf][n][kk + 2 * c + 8]);
            }
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) mma_bf16_16816(acc[i][j], af[i], bf[j]);
        }
        if (more) {
            stash(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }
    float* C = part + (size_t)blockIdx.z * M * N;
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int r = m0 + wm + i * 16 + g, n = n0 + wn + j * 8 + 2 * c;
            if (r < M) {
                if (n < N) C[(size_t)r * N + n] = acc[i][j][0];
                if (n + 1 < N) C[(size_t)r * N + n + 1] = acc[i][j][1];
            }
            if (r + 8 < M) {
                if (n < N) C[(size_t)(r + 8) * N + n] = acc[i][j][2];
                if (n + 1 < N) C[(size_t)(r + 8) * N + n + 1] = acc[i][j][3];
            }
        }
}

// One warp per token. A logits row holds E + 1 values (the last is the shared-gate logit) at row
// stride ld. The K chunks of the logits (ks of them, [ks][T][ld]) are summed in chunk order into
// chunk 0.
__global__ void router_topk_kernel(float* __restrict__ logits, int ld, const float* __restrict__ bias, int T, int E,
                                   int k, int ks, float* __restrict__ probs, int32_t* __restrict__ idx,
                                   float* __restrict__ w, float* __restrict__ sgate) {
    pdl_wait();
    pdl_launch_dependents();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    float* lg = logits + (size_t)warp * ld;
    for (int e = lane; e <= E; e += 32) {
        float part[kMaxKSplit];   // all chunk loads in flight at once, then summed in chunk order
#pragma unroll
        for (int z = 0; z < kMaxKSplit; ++z)
            part[z] = z < ks ? logits[(size_t)z * T * ld + (size_t)warp * ld + e] : 0.f;
        float v = part[0];
#pragma unroll
        for (int z = 1; z < kMaxKSplit; ++z)
            if (z < ks) v += part[z];
        if (bias && e < E) v += bias[e];
        lg[e] = v;
    }
    __syncwarp();
    float mx = -1e30f;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lg[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    double den = 0.0;
    for (int e = lane; e < E; e += 32) den += (double)expf(lg[e] - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    const float inv = (float)(1.0 / den);
    if (probs)
        for (int e = lane; e < E; e += 32) probs[(size_t)warp * E + e] = expf(lg[e] - mx) * inv;
    // top-k: k rounds of a warp arg-max over the untaken experts (p strictly greater wins; equal p
    // keeps the lower index). A lane owns experts lane, lane + 32, ...; `taken` bit i = expert lane+32i.
    uint32_t taken = 0;
    float ws[kMaxTopK];
    int ids[kMaxTopK];
    double wsum = 0.0;
    for (int s = 0; s < k; ++s) {
        float bp = -1.0f;
        int be = 0x7fffffff;
        for (int i = 0, e = lane; e < E; ++i, e += 32) {
            if (taken >> i & 1u) continue;
            const float p = expf(lg[e] - mx) * inv;
            if (p > bp) { bp = p; be = e; }   // ascending e within a lane: ties keep the lower index
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float op = __shfl_xor_sync(0xffffffffu, bp, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (op > bp || (op == bp && oe < be)) { bp = op; be = oe; }
        }
        if ((be & 31) == lane) taken |= 1u << (be >> 5);
        ids[s] = be;
        ws[s] = bp;
        wsum += (double)bp;
    }
    if (lane == 0) {
        for (int s = 0; s < k; ++s) {
            idx[(size_t)warp * k + s] = ids[s];
            w[(size_t)warp * k + s] = (float)((double)ws[s] / wsum);
        }
        if (sgate) sgate[warp] = 1.0f / (1.0f + expf(-lg[E]));
    }
}

// The same result for E <= 256, with each lane's (up to 8) probabilities kept in registers: the ks K
// chunks summed in chunk order (as above), one exp per expert, then k rounds of (lane max, warp arg-max).
// The shared-gate logit is the logits row's column E.
template <bool SPLIT>
__global__ void router_topk8_kernel(const float* __restrict__ logits, int ld, int ks, const float* __restrict__ bias,
                                    int T, int E, int k, float* __restrict__ probs, int32_t* __restrict__ idx,
                                    float* __restrict__ w, float* __restrict__ sgate) {
    pdl_wait();
    pdl_launch_dependents();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float* lg = logits + (size_t)warp * ld;
    const size_t zs = (size_t)T * ld;
    // the lane's eight logits and the shared-gate logit (slot 8), each summed over the ks K chunks in
    // chunk order (ks = 1 without SPLIT); the loads of four chunks for all nine are issued before their
    // adds, so the sums cost ceil(ks / 4) round trips to L2
    float s[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) s[i] = 0.f;
    for (int z0 = 0; z0 < ks; z0 += 4) {
        float pv[4][9];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < 9; ++i) {
                const int e = i < 8 ? lane + 32 * i : E;
                const bool on = z0 + u < ks && (i < 8 ? e < E : sgate != nullptr);
                pv[u][i] = on ? lg[(size_t)(z0 + u) * zs + e] : 0.f;
            }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < 9; ++i)
                if (z0 + u < ks) s[i] = z0 + u == 0 ? pv[u][i] : s[i] + pv[u][i];
    }
    const float gl = s[8];
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < E ? s[i] + (bias ? bias[e] : 0.f) : -INFINITY;
    }
    float mx = v[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, v[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    double den = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[i] = lane + 32 * i < E ? expf(v[i] - mx) : 0.f;   // e, then p below
        den += (double)v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    const float inv = (float)(1.0 / den);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[i] *= inv;
        if (probs && lane + 32 * i < E) probs[(size_t)warp * E + lane + 32 * i] = v[i];
    }
    // lane s keeps slot s's (expert, probability) in registers (k <= 16 < 32)
    float wsel = 0.f;
    int isel = 0;
    double wsum = 0.0;
    uint32_t taken = 0;
    for (int s = 0; s < k; ++s) {
        float bp = -1.0f;
        int be = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < 8; ++i)   // ascending e within a lane: ties keep the lower index
            if (!(taken >> i & 1u) && lane + 32 * i < E && v[i] > bp) { bp = v[i]; be = lane + 32 * i; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float op = __shfl_xor_sync(0xffffffffu, bp, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (op > bp || (op == bp && oe < be)) { bp = op; be = oe; }
        }
        if ((be & 31) == lane) taken |= 1u << (be >> 5);
        if (lane == s) { isel = be; wsel = bp; }
        wsum += (double)bp;
    }
    if (lane < k) {   // lane s writes slot s
        idx[(size_t)warp * k + lane] = isel;
        w[(size_t)warp * k + lane] = (float)((double)wsel / wsum);
    }
    if (lane == 0 && sgate) sgate[warp] = 1.0f / (1.0f + expf(-gl));
}

// Post-attention RMSNorm fused with the bf16 conversion, one warp per token: xb[t] = bf16(f32((x[t] /
// sqrt(mean(x[t]^2) + eps)) * w)) with the sum of squares, the rms, the division and the product in
// fp64 (Core::rmsnorm_host, src/open_qwen36/core.cpp:3014-3044, groups = 1; weight bf16).
__global__ void rmsnorm_bf16_kernel(const float* __restrict__ x, const uint16_t* __restrict__ w, double eps, int T, int H,
                                    uint16_t* __restrict__ xb) {
    pdl_wait();
    pdl_launch_dependents();
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (t >= T) return;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)t * H);
    double ss = 0.0;
    for (int i = lane; i < H / 4; i += 32) {
        const float4 v = xr[i];
        ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const double rms = sqrt(ss / (double)H + eps);
    const uint2* wr = reinterpret_cast<const uint2*>(w);
    uint2* o = reinterpret_cast<uint2*>(xb + (size_t)t * H);
    for (int i = lane; i < H / 4; i += 32) {
        const float4 v = xr[i];
        const uint2 ww = wr[i];
        const float a = (float)(((double)v.x / rms) * (double)__uint_as_float(ww.x << 16));
        const float b = (float)(((double)v.y / rms) * (double)__uint_as_float(ww.x & 0xFFFF0000u));
        const float c = (float)(((double)v.z / rms) * (double)__uint_as_float(ww.y << 16));
        const float d = (float)(((double)v.w / rms) * (double)__uint_as_float(ww.y & 0xFFFF0000u));
        o[i] = make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d));
    }
}

int launch_rmsnorm_bf16(const float* x, const uint16_t* w, float eps, int T, int H, uint16_t* xb, cudaStream_t st) {
    if (T <= 0) return FM_OK;
    FM_LAUNCH_PDL("rmsnorm_bf16", rmsnorm_bf16_kernel, dim3((T + 7) / 8), dim3(256), 0, st, x, w, (double)eps, T, H, xb);
    return FM_OK;
}

int launch_to_bf16(const float* x, uint16_t* xb, long long n, cudaStream_t st) {
    const long long n4 = n / 4;
    const int grid = (int)((n4 + 255) / 256 < 2048 ? (n4 + 255) / 256 : 2048);
    FM_LAUNCH_PDL("to_bf16", to_bf16_kernel, dim3(grid > 0 ? grid : 1), dim3(256), 0, st, x, xb, n4);
    return FM_OK;
}

// K chunks of the router GEMM: enough CTAs to cover the SMs when few tokens give few tiles. The logits
// rows hold E + 1 values (the last is the shared-gate logit).
size_t router_scratch_bytes(int T, int H, int E, bool fixed) {
    if (router_tc_ok(T, E, 1, fixed)) return (size_t)T * router_tc_ld(E) * 4;
    return (size_t)router_ksplit(T, H, E, fixed) * T * (E + 1) * 4;
}

int router_ksplit(int T, int H, int E, bool fixed) {
    if (fixed || T >= kRouterTcMinT) return 1;
    const int tiles = ((E + 1 + RG_BN - 1) / RG_BN) * ((T + RG_BM - 1) / RG_BM);
    int ks = 1;
    while (ks < kMaxKSplit && tiles * ks < 148 && H % (2 * ks * RG_BK) == 0) ks *= 2;
    return ks;
}

int launch_router(const uint16_t* xb, const uint16_t* router, const float* bias, int T, int H, int E, int k, bool fixed,
                  float* logits, float* probs, int32_t* idx, float* w, float* sgate, int* err, cudaStream_t st) {
    const bool tc = router_tc_ok(T, E, k, fixed);
    const int ks = tc ? 1 : router_ksplit(T, H, E, fixed);
    const int ld = tc ? router_tc_ld(E) : E + 1;
    if (tc) {
        if (int rc = launch_router_tc_logits(xb, router, T, H, E, logits, err, st)) return rc;
    } else {
        dim3 grid((E + 1 + RG_BN - 1) / RG_BN, (T + RG_BM - 1) / RG_BM, ks);
        FM_LAUNCH_PDL("router_logits", router_logits_kernel, grid, dim3(128), 0, st, xb, router, logits, T, E + 1, H);
    }
    if (E <= 256) {
        if (ks > 1)   // one warp per CTA: each token's ks x (E + 1) partial logits stream into its own SM
            FM_LAUNCH_PDL("router_topk8", router_topk8_kernel<true>, dim3(T), dim3(32), 0, st, logits, ld, ks, bias, T, E,
                          k, probs, idx, w, sgate);
        else
            FM_LAUNCH_PDL("router_topk8", router_topk8_kernel<false>, dim3((T + 7) / 8), dim3(256), 0, st, logits, ld, ks,
                          bias, T, E, k, probs, idx, w, sgate);
    } else {
        FM_LAUNCH_PDL("router_topk", router_topk_kernel, dim3((T + 7) / 8), dim3(256), 0, st, logits, ld, bias, T, E, k, ks,
                      probs, idx, w, sgate);
    }
    return FM_OK;
}

}  // namespace fm
