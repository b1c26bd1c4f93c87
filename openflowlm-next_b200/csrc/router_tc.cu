// Prefill-size router on the 5th-generation tensor cores, fused with the softmax top-k: one CTA per 128
// tokens computes the [128 x (E + 1)] logits of its tokens (the E router rows and the shared-expert gate
// row) into TMEM and turns them into the routing in the same kernel, so the logits never leave the SM.
//
//   warp 0     TMA producer: per 64-wide K slab, the 128 token rows of xb and the E + 1 router rows
//              (rows past E + 1, up to a multiple of 16, read as zeros), 4 stages;
//   warp 1     TMEM owner and MMA issuer: tcgen05.mma M = 128 tokens, N = E + 1 rounded up to 16 (two
//              MMAs when that is more than 256), K = 16, bf16 in, f32 accumulation;
//   warps 2-5  one thread per token (TMEM lane): max, softmax denominator and top-k over the token's
//              accumulator row, read back from TMEM 32 columns at a time.
//
// The routing follows host::router_block (src/open_qwen36/block_host.cpp:766-803) as the other router
// kernels do: logits + bias, max subtraction, float exp with a double denominator, p = e * float(1/den),
// top-k by probability with the lowest index on a tie (experts are taken in ascending order and a later
// one must be strictly larger to pass an earlier one), weights renormalised by a double sum; the
// shared-expert gate is sigmoid of the gate row's logit (core.cpp:4370-4373).
// Every mbarrier wait is bounded: a give-up records FM_ETIMEOUT in err[1] and the CTA drains and exits.
#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace fm {

constexpr int RT_BM = 128;                 // tokens per CTA (MMA M = TMEM lanes)
constexpr int RT_STAGES = 4;
constexpr int RT_A_BYTES = RT_BM * 128;    // 128 token rows x 64 bf16
constexpr int RT_THREADS = 192;

struct RouterTcArgs {
    const float* bias;
    int T, E, k;
    int ntot;        // MMA columns: E + 1 rounded up to 16 (<= 272)
    int nbox;        // router boxes per stage (1, or 2 when ntot > 256)
    int box_rows;    // rows per router box (ntot / nbox)
    int slabs;       // H / 64
    float* probs;
    int32_t* idx;
    float* w;
    float* sgate;
    int* err;
};

__host__ __device__ constexpr int rt_stage_bytes(int ntot) { return RT_A_BYTES + ntot * 128; }

// One (p, e) offered to a descending top list of k entries (ties: the earlier expert first). Experts
// arrive in ascending order, so the new one passes an entry only when strictly larger; once it has
// displaced an entry, the displaced one (earlier than every entry after it) passes equal entries.
// kth tracks tv[k - 1] (kept apart so that no register array is indexed at run time).
template <int KMAX>
__device__ __forceinline__ void topk_offer(float (&tv)[KMAX], int (&ti)[KMAX], float& kth, int k, float p, int e) {
    if (!(p > kth)) return;
    float cv = p;
    int ci = e;
    bool carried = false;
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
        if (j < k && (carried ? cv >= tv[j] : cv > tv[j])) {
            const float t = tv[j];
            const int u = ti[j];
            tv[j] = cv;
            ti[j] = ci;
            cv = t;
            ci = u;
            carried = true;
        }
    }
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
        if (j == k - 1) kth = tv[j];
}

template <int KMAX>
__global__ void __launch_bounds__(RT_THREADS, 1) router_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                   const __grid_constant__ CUtensorMap wmap, RouterTcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int stage_bytes = rt_stage_bytes(a.ntot);
    float* sbias = reinterpret_cast<float*>(smem + RT_STAGES * stage_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sbias + ((a.E + 3) & ~3));
    uint64_t* full = bars;
    uint64_t* empty = full + RT_STAGES;
    uint64_t* acc_full = empty + RT_STAGES;
    uint64_t* drain = acc_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * RT_BM;
    for (int e = threadIdx.x; e < a.E; e += RT_THREADS) sbias[e] = a.bias ? a.bias[e] : 0.f;
    if (threadIdx.x == 0) {
        for (int i = 0; i < RT_STAGES; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        mbar_init(acc_full, 1);
        mbar_init(drain, 1);
        mbar_fence_init();
        prefetch_tmap(&xmap);
        prefetch_tmap(&wmap);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            int st = 0;
            uint32_t ph = 0, issued = 0;
            bool ok = true;
            for (int s = 0; s < a.slabs; ++s) {
                if (!mbar_wait(&empty[st], ph ^ 1)) { ok = false; break; }
                mbar_expect_tx(&full[st], stage_bytes);
                uint8_t* A = smem + st * stage_bytes;
                tma_load_2d(A, &xmap, s * 64, m0, &full[st]);
                for (int j = 0; j < a.nbox; ++j)
                    tma_load_2d(A + RT_A_BYTES + j * a.box_rows * 128, &wmap, s * 64, j * a.box_rows, &full[st]);
                issued |= 1u << st;
                if (++st == RT_STAGES) { st = 0; ph ^= 1; }
            }
            if (!ok) {
                atomicCAS(a.err + 1, 0, FM_ETIMEOUT);
                for (int i = 0; i < RT_STAGES; ++i) {   // every slot's latest fill lands before the CTA exits
                    const int slot = (st + i) % RT_STAGES;
                    if (issued >> slot & 1u) mbar_wait(&full[slot], slot < st ? ph : ph ^ 1);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const int n1 = a.ntot < 256 ? a.ntot : 256;
            const uint32_t id1 = idesc_bf16(RT_BM, n1);
            const uint32_t id2 = a.ntot > 256 ? idesc_bf16(RT_BM, a.ntot - 256) : 0u;
            int st = 0;
            uint32_t ph = 0;
            bool ok = true, any = false;
            for (int s = 0; s < a.slabs; ++s) {
                if (!mbar_wait(&full[st], ph)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + st * stage_bytes);
                const uint32_t sb = sa + RT_A_BYTES;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t acc = (s > 0 || kk > 0) ? 1u : 0u;
                    tc_mma_f16(tmem_base, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + kk * 32), id1, acc);
                    if (a.ntot > 256)
                        tc_mma_f16(tmem_base + 256, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + 256 * 128 + kk * 32), id2,
                                   acc);
                }
                any = true;
                tc_commit(&empty[st]);
                if (++st == RT_STAGES) { st = 0; ph ^= 1; }
            }
            if (ok) tc_commit(acc_full);
            else atomicCAS(a.err + 1, 0, FM_ETIMEOUT);
            if (any) {   // every MMA complete before TMEM is released
                tc_commit(drain);
                mbar_wait(drain, 0);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue: one thread per token
        const int lg = warp & 3;                     // the TMEM lane quarter this warp may read
        const int row = lg * 32 + lane;
        const int t = m0 + row;
        const bool live = t < a.T;
        const bool ok = mbar_wait(acc_full, 0);
        if (!ok) atomicCAS(a.err + 1, 0, FM_ETIMEOUT);
        if (__all_sync(0xffffffffu, ok)) {
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(lg * 32) << 16);
            const int E = a.E, k = a.k;
            float mx = -INFINITY;
            for (int c0 = 0; c0 < E; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (c0 + j < E) mx = fmaxf(mx, __uint_as_float(v[j]) + sbias[c0 + j]);
            }
            double den = 0.0;
            for (int c0 = 0; c0 < E; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (c0 + j < E) den += (double)expf(__uint_as_float(v[j]) + sbias[c0 + j] - mx);
            }
            const float inv = (float)(1.0 / den);
            float tv[KMAX];
            int ti[KMAX];
#pragma unroll
            for (int j = 0; j < KMAX; ++j) { tv[j] = -1.0f; ti[j] = 0x7fffffff; }
            float kth = -1.0f;
            float* prow = (a.probs && live) ? a.probs + (size_t)t * E : nullptr;
            for (int c0 = 0; c0 < E; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int e = c0 + j;
                    if (e < E) {
                        const float p = expf(__uint_as_float(v[j]) + sbias[e] - mx) * inv;
                        topk_offer<KMAX>(tv, ti, kth, k, p, e);
                        if (prow) prow[e] = p;
                    }
                }
            }
            if (a.sgate) {   // the gate row's logit: column E
                uint32_t v[32];
                tmem_ld32(taddr + (E & ~31), v);
                tmem_ld_wait();
                float gl = 0.f;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j == (E & 31)) gl = __uint_as_float(v[j]);
                if (live) a.sgate[t] = 1.0f / (1.0f + expf(-gl));
            }
            if (live) {
                double wsum = 0.0;
#pragma unroll
                for (int s = 0; s < KMAX; ++s)
                    if (s < k) wsum += (double)tv[s];
#pragma unroll
                for (int s = 0; s < KMAX; ++s) {
                    if (s < k) {
                        a.idx[(size_t)t * k + s] = ti[s];
                        a.w[(size_t)t * k + s] = (float)((double)tv[s] / wsum);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

bool router_tc_ok(int T, int E, int k) { return T >= kRouterTcMinT && E + 1 <= 272 && k <= kMaxTopK; }

int launch_router_tc(const uint16_t* xb, const uint16_t* router, const float* bias, int T, int H, int E, int k,
                     float* probs, int32_t* idx, float* w, float* sgate, int* err, cudaStream_t st) {
    RouterTcArgs a{};
    a.bias = bias;
    a.T = T;
    a.E = E;
    a.k = k;
    a.ntot = (E + 1 + 15) / 16 * 16;
    a.nbox = (a.ntot + 255) / 256;
    a.box_rows = a.ntot / a.nbox;
    a.slabs = H / 64;
    a.probs = probs;
    a.idx = idx;
    a.w = w;
    a.sgate = sgate;
    a.err = err;
    CUtensorMap xmap, wmap;
    if (int rc = make_bmap(&xmap, xb, T, H, H, RT_BM)) return rc;
    if (int rc = make_bmap(&wmap, router, E + 1, H, H, a.box_rows)) return rc;
    const int smem = RT_STAGES * rt_stage_bytes(a.ntot) + ((E + 3) & ~3) * 4 + 8 * (2 * RT_STAGES + 2) + 16 + 1024;
    const int grid = (T + RT_BM - 1) / RT_BM;
    cudaError_t e;
    if (k <= 8) {
        if ((e = raise_smem_limit((const void*)router_tc_kernel<8>, smem))) return cuda_status(e, "router_tc smem");
        router_tc_kernel<8><<<grid, RT_THREADS, smem, st>>>(xmap, wmap, a);
    } else {
        if ((e = raise_smem_limit((const void*)router_tc_kernel<16>, smem))) return cuda_status(e, "router_tc smem");
        router_tc_kernel<16><<<grid, RT_THREADS, smem, st>>>(xmap, wmap, a);
    }
    FM_LAUNCH_CHECK("router_tc");
    return FM_OK;
}

}  // namespace fm
