// Prefill-size router logits on the 5th-generation tensor cores: logits[t][0..E] = xb[t] . router[0..E]
// (the E router rows and the shared-expert gate row) in f32, for the router_topk8 kernel that follows.
// CTA (token tile of 128, column half): a tile's two CTAs each take half of the E + 1 columns (rounded
// to 16), so a 8192-token call runs on 128 CTAs, and the second reads the tile's activations from L2.
//
//   warp 0     TMA producer: per 64-wide K slab, the 128 token rows of xb and the CTA's router rows (rows
//              past E + 1 read as zeros), 4 stages;
//   warp 1     TMEM owner and MMA issuer: tcgen05.mma M = 128 tokens, N = the CTA's columns, K = 16, bf16
//              in, f32 accumulation;
//   warps 2-5  epilogue: thread = token (TMEM lane), 32 columns per tcgen05.ld, 16-byte stores of its
//              logits row segment (row stride ld, a multiple of 4).
//
// The top-k of each token (softmax, lowest index on a tie, renormalised; host::router_block,
// src/open_qwen36/block_host.cpp:766-803) runs in router_topk8 with one warp per token: routing 128
// tokens inside this CTA would serialise 128 dependent shuffle chains on four warps.
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
    int T, E;
    int ncols;       // MMA columns of one CTA (a multiple of 16, <= 256)
    int slabs;       // H / 64
    float* logits;   // [T, ld] f32
    int ld;
    int* err;
};

__host__ __device__ constexpr int rt_stage_bytes(int ntot) { return RT_A_BYTES + ntot * 128; }

__global__ void __launch_bounds__(RT_THREADS, 1) router_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                   const __grid_constant__ CUtensorMap wmap, RouterTcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int stage_bytes = rt_stage_bytes(a.ncols);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + RT_STAGES * stage_bytes);
    uint64_t* full = bars;
    uint64_t* empty = full + RT_STAGES;
    uint64_t* acc_full = empty + RT_STAGES;
    uint64_t* drain = acc_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = (blockIdx.x >> 1) * RT_BM;           // the token tile
    const int n0 = (blockIdx.x & 1) * a.ncols;          // the CTA's first column
    if (threadIdx.x == 0) {
        for (int i = 0; i < RT_STAGES; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        mbar_init(acc_full, 1);
        mbar_init(drain, 1);
        mbar_fence_init();
        prefetch_tmap(&xmap);
        prefetch_tmap(&wmap);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 256);
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
                tma_load_2d(A + RT_A_BYTES, &wmap, s * 64, n0, &full[st]);
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
            const uint32_t idesc = idesc_bf16(RT_BM, a.ncols);
            int st = 0;
            uint32_t ph = 0;
            bool ok = true, any = false;
            for (int s = 0; s < a.slabs; ++s) {
                if (!mbar_wait(&full[st], ph)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + st * stage_bytes);
                const uint32_t sb = sa + RT_A_BYTES;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    tc_mma_f16(tmem_base, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + kk * 32), idesc,
                               (s > 0 || kk > 0) ? 1u : 0u);
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
        // ---------------------------------------------------------------- epilogue: thread = token
        const int lg = warp & 3;                     // the TMEM lane quarter this warp may read
        const int t = m0 + lg * 32 + lane;
        const bool ok = mbar_wait(acc_full, 0);
        if (!ok) atomicCAS(a.err + 1, 0, FM_ETIMEOUT);
        if (__all_sync(0xffffffffu, ok)) {
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(lg * 32) << 16);
            const int ncols = min(a.ncols, a.E + 1 - n0);   // this CTA's real columns
            float* row = a.logits + (size_t)t * a.ld + n0;
            for (int c0 = 0; c0 < ncols; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                tmem_ld_wait();
                if (t < a.T) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        if (c0 + j + 4 <= ncols) {
                            *reinterpret_cast<float4*>(row + c0 + j) = make_float4(
                                __uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                __uint_as_float(v[j + 3]));
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if (c0 + j + q < ncols) row[c0 + j + q] = __uint_as_float(v[j + q]);
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 256);
    }
}

bool router_tc_ok(int T, int E, int k, bool fixed) {
    return (fixed || T >= kRouterTcMinT) && E <= 496 && k <= kMaxTopK;
}

int router_tc_ld(int E) { return (E + 1 + 3) & ~3; }

int launch_router_tc_logits(const uint16_t* xb, const uint16_t* router, int T, int H, int E, float* logits, int* err,
                            cudaStream_t st) {
    RouterTcArgs a{};
    a.T = T;
    a.E = E;
    a.ncols = ((E + 1 + 1) / 2 + 15) / 16 * 16;   // half of E + 1, rounded up to 16
    a.slabs = H / 64;
    a.logits = logits;
    a.ld = router_tc_ld(E);
    a.err = err;
    CUtensorMap xmap, wmap;
    if (int rc = make_bmap(&xmap, xb, T, H, H, RT_BM)) return rc;
    if (int rc = make_bmap(&wmap, router, E + 1, H, H, a.ncols)) return rc;
    const int smem = RT_STAGES * rt_stage_bytes(a.ncols) + 8 * (2 * RT_STAGES + 2) + 16 + 1024;
    const int grid = 2 * ((T + RT_BM - 1) / RT_BM);
    if (cudaError_t e = raise_smem_limit((const void*)router_tc_kernel, smem)) return cuda_status(e, "router_tc smem");
    router_tc_kernel<<<grid, RT_THREADS, smem, st>>>(xmap, wmap, a);
    FM_LAUNCH_CHECK("router_tc");
    return FM_OK;
}

}  // namespace fm
