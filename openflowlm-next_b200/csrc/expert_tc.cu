// Grouped Q4_1 expert GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// One persistent CTA per SM walks the work list (group, band, first sorted row, rows). A work item
// is D[128 weight rows x n tokens] = W_band[128 x K] . X[n x K]^T with n <= 256, K walked in 64-wide
// slabs. Warp roles (480 threads for gate_up, 608 for down):
//   warp 0      weight producer: per slab, one 5120-byte bulk copy of the raw Q4_1 weight tile;
//   last warp   activation producer: per slab, 128- and 32-row TMA loads (128-byte swizzle) of the
//               sorted bf16 activation rows;
//   warp 1      TMEM owner and MMA issuer: four tcgen05.mma (M=128, N=n rounded to 16, K=16) per
//               slab into one of two TMEM accumulators (2 x 256 columns), commits release the rings;
//   warps 2-9   dequantisers, two groups taking alternate slabs: thread r of a group turns row r of
//               the raw tile (two GGUF blocks) into 64 bf16
//               values in the 128-byte-swizzled K-major layout the MMA reads (w = q*d + m in f32 with
//               the fp16 d, m widened exactly, rounded once to bf16);
//   warps 10-   epilogue (gate_up 4 warps; down 8 in two halves taking alternate 32-token chunks),
//               overlapped with the next item's main loop through the second accumulator:
//               GATE_UP  rows 0-63 of a gate_up tile are gate rows, rows 64-127 the up rows of the same
//                        64 features: h = bf16(silu(g) * u) -> the sorted h matrix (the reference's
//                        SwiGLU, designs/moe_batch/moe_batch.h:181-202, h rounded to bf16);
//               DOWN     out[token][row] += w * y (the weighted scatter of core.cpp:5236-5255, routing
//                        weight or shared-expert gate per row): the weighted 32-token chunk is staged
//                        in shared memory, then each warp adds 8 token rows with red.global.add.v4.f32;
//                        or unweighted bf16 y rows (expert parallel: in the received order, or straight
//                        into the sending rank's buffer over peer memory).
// Every mbarrier wait is bounded (sm100.cuh); a give-up records FM_ETIMEOUT in the error word and
// the CTA drains its own copies, frees TMEM and returns.
#include <cuda.h>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace fm {

// Warp roles: 0 weight producer, 1 MMA issuer, then DQ dequantiser warps (groups of 4 working alternate
// slabs), EPI epilogue warps (groups of 4, "halves", taking alternate 32-token chunks), and the
// activation producer last. gate_up (K = H = 2048, light epilogue): 8 + 4, 480 threads; down
// (K = F = 512, a y row per token and band): 8 + 8, 608 threads.
template <bool GATE_UP>
struct TcRoles {
    static constexpr int DQ = 8;
    static constexpr int EPI = GATE_UP ? 4 : 8;
    static constexpr int EPI0 = 2 + DQ;          // first epilogue warp
    static constexpr int BWARP = EPI0 + EPI;     // activation producer warp
    static constexpr int THREADS = 32 * (BWARP + 1);
};
constexpr int TC_BOX_BIG = 128;            // activation rows per large TMA box
constexpr int TC_BN = 256;                 // max tokens per work item (MMA N)
constexpr int TC_A_BYTES = 128 * 128;      // 128 rows x 64 bf16
constexpr int TC_B_BYTES = TC_BN * 128;    // 256 rows x 64 bf16
constexpr int TC_BOX_ROWS = 32;
constexpr int TC_EPI_LD = 132;             // padded f32 row of the DOWN staging tile
// epilogue staging: GATE_UP gate/up exchange (2 x 16 x 64 f32) + h tile (32 x 64 bf16);
// DOWN weighted y tile (32 x 132 f32) + token / weight lists (2 x 256)
constexpr int TC_HALF_BYTES = 32 * TC_EPI_LD * 4;            // one epilogue half's staging area
constexpr int TC_EPI_BYTES = 2 * TC_HALF_BYTES + 2 * 256 * 4;   // two halves + token / weight lists

// Shared-memory layout. gate_up (K = 2048: 32 slabs per item, a light epilogue): 4 dequantised A stages,
// 4 raw weight tiles, the gate/up exchange and h staging of one epilogue half (12 KB); down (K = 512, two
// epilogue halves with 32 x 132 f32 staging each and the token / weight lists): 2 A stages, 6 raw tiles.
// Both: 128 KB of activation stages (4 of 256 rows for one CTA per item, 8 of 128 rows for a CTA-pair
// member). Two dequantiser groups take alternate slabs, so with 4 A stages each group has a second
// stage to fill while the tensor core still reads its first.
template <bool GATE_UP, bool PAIR>
struct TcSmem {
    static constexpr int SA = GATE_UP ? 4 : 2;
    static constexpr int SB = PAIR ? 8 : 4;
    static constexpr int SR = GATE_UP ? 4 : 6;    // raw weight tiles in flight (streamed from HBM)
    static constexpr int B_STAGE = PAIR ? TC_B_BYTES / 2 : TC_B_BYTES;
    static constexpr int EPI = GATE_UP ? 3 * 16 * 64 * 4 : TC_EPI_BYTES;
    // offsets from the 1024-aligned dynamic smem base
    static constexpr int a = 0;
    static constexpr int b = a + SA * TC_A_BYTES;
    static constexpr int raw = b + SB * B_STAGE;
    static constexpr int epi = raw + SR * kTileBytes;
    static constexpr int bars = epi + EPI;
    // raw, activation, A and accumulator rings + drain
    static constexpr int nbars = 2 * SR + 2 * SB + 2 * SA + 4 + 1;
    static constexpr int tmem = bars + nbars * 8;
    static constexpr int total = tmem + 16 + 1024;   // + alignment slack
};
static_assert(TcSmem<true, true>::total <= 232448 && TcSmem<true, false>::total <= 232448 &&
                  TcSmem<false, true>::total <= 232448 && TcSmem<false, false>::total <= 232448,
              "shared memory per CTA");

struct TcArgs {
    const int* list;
    const uint8_t* w_routed;
    size_t w_routed_stride;
    const uint8_t* w_shared;
    int shared_group;
    int K_routed, K_shared;
    // GATE_UP
    uint16_t* h_out;
    int h_ld;
    // DOWN
    float* out;
    int H;
    const int* pair;
    const float* wpair;
    int k;
    int shared_base;
    const float* sgate;
    // DOWN, row mode: routed row r's y, unweighted bf16, goes to y_rows[ymap ? ymap[r] : r]; without ymap
    // the shared expert's rows go to y_rows[r] too (a combine kernel then sums each token in ascending
    // expert order), with ymap they are added into out (expert parallel: out holds this rank's tokens)
    uint16_t* y_rows;
    const int* ymap;
    // DOWN, peer expert-parallel mode: routed row r's y, unweighted bf16, goes straight to the rank that
    // sent the row: yret[meta[r] >> 24] + (meta[r] & 0xFFFFFF) rows, a store over NVLink; skipped once
    // the status word *err is set (a failed exchange: the peers may be gone)
    const int* meta;
    uint16_t* yret[kMaxRanks];
    int* err;
};

__device__ __forceinline__ void fail(int* err, int code) { atomicCAS(err, 0, code); }

// Code q (0..15, byte b of t) as the float 0.5 + q/256: a byte permute places q in mantissa bits
// 16-19 under the exponent byte 0x3F. Then q*d + m = f * (256 d) + (m - 128 d): the product is exact
// (8 x 11 significant bits) and the single rounding of the add is the only one besides the fp32
// rounding of the per-block constant m - 128 d (relative 2^-24), far below the bf16 rounding that
// follows.
__device__ __forceinline__ float code_f(uint32_t t, uint32_t sel) { return __uint_as_float(__byte_perm(t, 0x3F000000u, sel)); }

// Four codes (bytes of t) -> two bf16x2 words of q*d + m, with D = 256 d and C = m - 128 d.
__device__ __forceinline__ uint2 deq4(uint32_t t, float D, float C) {
    const float a = fmaf(code_f(t, 0x7044), D, C);
    const float b = fmaf(code_f(t, 0x7144), D, C);
    const float c = fmaf(code_f(t, 0x7244), D, C);
    const float e = fmaf(code_f(t, 0x7344), D, C);
    return make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, e));
}

// One GGUF block's 16 nibble bytes (4 words) -> 4 chunks of 8 bf16 (K = 0-7, 8-15, 16-23, 24-31).
__device__ __forceinline__ void deq_block(uint4 n, float d, float m, uint4* ch) {
    const float D = 256.0f * d, C = fmaf(-128.0f, d, m);
    const uint32_t w[4] = {n.x, n.y, n.z, n.w};
    uint2 lo[4], hi[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo[i] = deq4(w[i] & 0x0F0F0F0Fu, D, C);
        hi[i] = deq4((w[i] >> 4) & 0x0F0F0F0Fu, D, C);
    }
    ch[0] = make_uint4(lo[0].x, lo[0].y, lo[1].x, lo[1].y);   // values 0-7: low nibbles of bytes 0-7
    ch[1] = make_uint4(lo[2].x, lo[2].y, lo[3].x, lo[3].y);   // values 8-15
    ch[2] = make_uint4(hi[0].x, hi[0].y, hi[1].x, hi[1].y);   // values 16-23: high nibbles of bytes 0-7
    ch[3] = make_uint4(hi[2].x, hi[2].y, hi[3].x, hi[3].y);   // values 24-31
}

// A tile block's 4 words in fragment order (see repack.cu) -> GGUF byte order b0..b15.
__device__ __forceinline__ uint4 gguf_order(uint4 t) {
    return make_uint4(__byte_perm(t.x, t.y, 0x5410), __byte_perm(t.z, t.w, 0x5410), __byte_perm(t.x, t.y, 0x7632),
                      __byte_perm(t.z, t.w, 0x7632));
}

struct Item {
    int g, band, row0, n, slabs;
    const uint8_t* w;
};

// PAIR: list entries name band pairs; CTA `crank` of the pair takes band 2 * entry + crank.
template <bool PAIR>
__device__ __forceinline__ Item decode_item(const TcArgs& a, int i, uint32_t crank) {
    const int4 it = reinterpret_cast<const int4*>(a.list + 4)[i];
    Item r;
    r.g = it.x;
    r.band = PAIR ? 2 * it.y + (int)crank : it.y;
    r.row0 = it.z;
    r.n = it.w;
    const bool sh = r.g == a.shared_group;
    const int K = sh ? a.K_shared : a.K_routed;
    r.slabs = K / kTileK;
    const uint8_t* base = sh ? a.w_shared : a.w_routed + (size_t)r.g * a.w_routed_stride;
    r.w = base + (size_t)r.band * r.slabs * kTileBytes;
    return r;
}

// PAIR: a cluster of two CTAs on two SMs works each item as one M = 256 MMA (tcgen05 cta_group::2):
// CTA r dequantises band 2p + r into its own A ring and loads rows [r N/2, (r + 1) N/2) of the
// item's tokens into its own B ring, so each SM streams half the activation bytes per MMA. The first
// CTA's barriers gate the MMAs: its A-full barrier counts one arrival per dequantiser warp of both
// CTAs, its B-full barrier the bytes of both CTAs' activation loads (the second CTA's loads complete
// on it directly), its accumulator-empty barrier one arrival per epilogue warp of both CTAs; the
// first CTA issues the MMAs and commits the stage / accumulator releases to both CTAs' barriers. No
// load is shared between the CTAs and no multicast copy is used.
template <bool GATE_UP, bool PAIR>
__global__ void __launch_bounds__(TcRoles<GATE_UP>::THREADS, 1) expert_tc_kernel(const __grid_constant__ CUtensorMap bmap,
                                                                  const __grid_constant__ CUtensorMap bmap_big, TcArgs a) {
    using R = TcRoles<GATE_UP>;
    using Sm = TcSmem<GATE_UP, PAIR>;
    constexpr int SA = Sm::SA, SB = Sm::SB, SR = Sm::SR, B_STAGE = Sm::B_STAGE;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Sm::bars);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = raw_full + SR;
    uint64_t* b_full = raw_empty + SR;
    uint64_t* b_empty = b_full + SB;
    uint64_t* a_full = b_empty + SB;
    uint64_t* a_empty = a_full + SA;
    uint64_t* acc_full = a_empty + SA;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;             // the MMA issuer's last commit
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Sm::tmem);
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = a.list[0];
    const uint32_t crank = PAIR ? cluster_ctarank() : 0;
    const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;   // item stride: one per CTA or pair
    const int n_units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        // a dequantiser group (4 warps, 128 threads) consumes a raw tile and fills an A stage
        for (int i = 0; i < SR; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], 128); }
        for (int i = 0; i < SB; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
        // arrivals are per warp: 4 dequantiser / 4 or 8 epilogue warps per CTA, both CTAs' on the first CTA's
        for (int i = 0; i < SA; ++i) { mbar_init(&a_full[i], (PAIR ? 2 : 1) * 4); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], (PAIR ? 2 : 1) * R::EPI); }
        mbar_init(drain, 1);
        mbar_fence_init();
        prefetch_tmap(&bmap);
        prefetch_tmap(&bmap_big);
    }
    if (warp == 1) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, 512);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, 512);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if (PAIR) cluster_sync();   // barriers initialised in both CTAs before any cross-CTA arrival
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0 || warp == R::BWARP) {
        // ------------------------------------------------------------ producers (lane 0 of each)
        // warp 0: the raw weight tiles (streamed from HBM, SR deep); warp R::BWARP: the activation
        // rows (TMA, SB deep). Separate threads, so the weight stream runs ahead of the activations.
        const bool weights = warp == 0;
        if (lane == 0) {
            const int S = weights ? SR : SB;
            uint64_t* full = weights ? raw_full : b_full;
            uint64_t* empty = weights ? raw_empty : b_empty;
            int st = 0;
            uint32_t ph = 0, issued = 0;   // bit i: slot i has a fill in flight or landed
            bool ok = true;
            for (int i = unit; i < n_items && ok; i += n_units) {
                const Item it = decode_item<PAIR>(a, i, crank);
                // this CTA's token rows: all n (single), or its half of N = n rounded up to 16 (pair)
                const int nhalf = PAIR ? ((it.n + 15) & ~15) / 2 : it.n;
                const int rbase = it.row0 + (int)crank * nhalf;
                // whole 128-row boxes, then 32-row boxes for the rest
                const int nbig = nhalf / TC_BOX_BIG;
                const int nsmall = (nhalf - nbig * TC_BOX_BIG + TC_BOX_ROWS - 1) / TC_BOX_ROWS;
                const int rows_loaded = nbig * TC_BOX_BIG + nsmall * TC_BOX_ROWS;
                for (int s = 0; s < it.slabs; ++s) {
                    if (!mbar_wait(&empty[st], ph ^ 1)) { ok = false; break; }
                    if (weights) {
                        mbar_expect_tx(&raw_full[st], kTileBytes);
                        bulk_load(smem + Sm::raw + st * kTileBytes, it.w + (size_t)s * kTileBytes, kTileBytes, &raw_full[st]);
                        issued |= 1u << st;
                    } else {
                        // the first CTA arms its B-full barrier for both halves; the second CTA's loads
                        // complete their bytes on that barrier
                        if (crank == 0) mbar_expect_tx(&b_full[st], (PAIR ? 2 : 1) * rows_loaded * 128);
                        for (int j = 0; j < nbig + nsmall; ++j) {
                            const bool big = j < nbig;
                            const int r0 = big ? j * TC_BOX_BIG : nbig * TC_BOX_BIG + (j - nbig) * TC_BOX_ROWS;
                            const CUtensorMap* map = big ? &bmap_big : &bmap;
                            uint8_t* dst = smem + Sm::b + st * B_STAGE + r0 * 128;
                            if (PAIR)
                                tma_load_2d_pair(dst, map, s * kTileK, rbase + r0, mapa_shared(&b_full[st], 0));
                            else
                                tma_load_2d(dst, map, s * kTileK, rbase + r0, &b_full[st]);
                        }
                        if (crank == 0) issued |= 1u << st;
                    }
                    if (++st == S) { st = 0; ph ^= 1; }
                }
            }
            if (!ok) {
                fail(a.err, FM_ETIMEOUT);
                atomicExch(&abort_flag, 1);
                // drain: every slot's most recent fill must land before the CTA may exit
                for (int i = 0; i < S; ++i) {
                    const int slot = (st + i) % S;
                    const uint32_t p = slot < st ? ph : ph ^ 1;   // parity of the slot's last fill
                    if (issued >> slot & 1u) mbar_wait(&full[slot], p);
                }
            }
        }
    } else if (warp == 1) {
        if (!PAIR || crank == 0) {
            // -------------------------------------------------------- MMA issuer (first CTA of a pair)
            if (lane == 0) {
                int as = 0, bs = 0;
                uint32_t aph = 0, bph = 0;
                bool ok = true, issued = false;
                int local = 0;
                const uint32_t peer = 1;
                for (int i = unit; i < n_items && ok; i += n_units, ++local) {
                    const Item it = decode_item<PAIR>(a, i, crank);
                    const int acc = local & 1;
                    const uint32_t accph = (local >> 1) & 1;
                    if (!mbar_wait_cluster(&acc_empty[acc], accph ^ 1)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * 256;
                    const int N = (it.n + 15) & ~15;
                    const uint32_t idesc = idesc_bf16(PAIR ? 256 : 128, N);
                    for (int s = 0; s < it.slabs; ++s) {
                        if (!mbar_wait_cluster(&a_full[as], aph) || !mbar_wait(&b_full[bs], bph)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t sa = smem_u32(smem + Sm::a + as * TC_A_BYTES);
                        const uint32_t sb = smem_u32(smem + Sm::b + bs * B_STAGE);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            if (PAIR)
                                tc_mma_f16_pair(d_tmem, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + kk * 32), idesc,
                                                (s > 0 || kk > 0) ? 1u : 0u);
                            else
                                tc_mma_f16(d_tmem, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + kk * 32), idesc,
                                           (s > 0 || kk > 0) ? 1u : 0u);
                        }
                        issued = true;
                        if (PAIR) {   // both CTAs' stages are free once these MMAs completed
                            tc_commit_pair(mapa_shared(&a_empty[as], 0));
                            tc_commit_pair(mapa_shared(&a_empty[as], peer));
                            tc_commit_pair(mapa_shared(&b_empty[bs], 0));
                            tc_commit_pair(mapa_shared(&b_empty[bs], peer));
                        } else {
                            tc_commit(&a_empty[as]);
                            tc_commit(&b_empty[bs]);
                        }
                        if (++as == SA) { as = 0; aph ^= 1; }
                        if (++bs == SB) { bs = 0; bph ^= 1; }
                    }
                    if (!ok) break;
                    if (PAIR) {
                        tc_commit_pair(mapa_shared(&acc_full[acc], 0));
                        tc_commit_pair(mapa_shared(&acc_full[acc], peer));
                    } else {
                        tc_commit(&acc_full[acc]);
                    }
                }
                if (!ok) {
                    fail(a.err, FM_ETIMEOUT);
                    atomicExch(&abort_flag, 1);
                }
                // every MMA of this CTA (and its commits' arrivals) done before the pair may exit
                if (issued) {
                    if (PAIR) tc_commit_pair(mapa_shared(drain, 0));
                    else tc_commit(drain);
                    mbar_wait(drain, 0);
                }
            }
        }
    } else if (warp < R::EPI0) {
        // ------------------------------------------------------------ dequantisers
        // Groups of 4 warps; group g takes the slabs whose running index sc has sc % NG == g, so NG
        // slabs are dequantised at once (the per-slab chain of barrier, shared loads and stores is
        // latency-bound). Thread t of a group rebuilds row t of the tile (both 32-value blocks).
        constexpr int NG = R::DQ / 4;
        const int t = threadIdx.x - 64;
        const int grp = t >> 7;
        const int r = t & 127;
        bool ok = true;
        int sc = 0;   // running slab index over this CTA's items
        for (int i = unit; i < n_items && ok; i += n_units) {
            const Item it = decode_item<PAIR>(a, i, crank);
            for (int s = 0; s < it.slabs; ++s, ++sc) {
                if (sc % NG != grp) continue;
                const int rs = sc % SR, as = sc % SA;
                const uint32_t rph = (sc / SR) & 1, aph = (sc / SA) & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[rs], rph))) { ok = false; break; }
                const uint32_t raw = smem_u32(smem + Sm::raw + rs * kTileBytes);
                const uint4 n0 = gguf_order(lds128(raw + r * 32));
                const uint4 n1 = gguf_order(lds128(raw + r * 32 + 16));
                const uint2 sc2 = lds64(raw + kTileNibBytes + r * 8);
                const float d0 = __half2float(__ushort_as_half((unsigned short)(sc2.x & 0xFFFF)));
                const float m0 = __half2float(__ushort_as_half((unsigned short)(sc2.x >> 16)));
                const float d1 = __half2float(__ushort_as_half((unsigned short)(sc2.y & 0xFFFF)));
                const float m1 = __half2float(__ushort_as_half((unsigned short)(sc2.y >> 16)));
                uint4 ch[8];
                deq_block(n0, d0, m0, ch);
                deq_block(n1, d1, m1, ch + 4);
                // The raw slot goes back to the weight producer, whose next bulk copy (async proxy)
                // overwrites it, only after this thread's loads from it have delivered their values (the
                // dequantised words depend on them) and a proxy fence: releasing it right after issuing
                // the loads let the copy land under loads still in flight on B200 (wrong weights for a
                // slab, intermittently).
                fence_proxy_async_smem();
                mbar_arrive(&raw_empty[rs]);
                if (!__all_sync(0xffffffffu, mbar_wait(&a_empty[as], aph ^ 1))) { ok = false; break; }
                const uint32_t arow = smem_u32(smem + Sm::a + as * TC_A_BYTES + r * 128);
#pragma unroll
                for (int c = 0; c < 8; ++c) sts128(arow + ((c ^ (r & 7)) << 4), ch[c]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {   // the warp's 32 rows are in place (on the first CTA's barrier)
                    if (PAIR && crank == 1) mbar_arrive_cluster(mapa_shared(&a_full[as], 0));
                    else mbar_arrive(&a_full[as]);
                }
            }
        }
        if (!ok) {
            fail(a.err, FM_ETIMEOUT);
            atomicExch(&abort_flag, 1);
        }
    } else {
        // ------------------------------------------------------------ epilogue (4 or 8 warps)
        // Warp w reads TMEM lane group w % 4. With 8 warps, the half (w - EPI0) / 4 takes every other
        // 32-column chunk (c0 = 32 half + 64 i) with its own staging area and named barrier (1 + half,
        // 128 threads); barrier 3 spans all epilogue threads.
        constexpr int HALVES = R::EPI / 4;
        const int lg = warp & 3;                 // TMEM lane group this warp may access
        const int row = lg * 32 + lane;          // accumulator row = TMEM lane
        const int et = threadIdx.x - 32 * R::EPI0;   // 0 .. 32 EPI - 1
        const int half = et >> 7;
        const int ht = et & 127;                 // thread within the half
        const int hbar = 1 + half;
        uint8_t* epi = smem + Sm::epi + half * TC_HALF_BYTES;
        float* xg = reinterpret_cast<float*>(epi);                   // GATE_UP: gate, cols 16-31 [16][64]
        float* xu = xg + 16 * 64;                                    //          up, cols 0-15 [16][64]
        uint16_t* hst = reinterpret_cast<uint16_t*>(xu + 16 * 64);   //          h tile [32][64] bf16
        float* ys = reinterpret_cast<float*>(epi);                   // DOWN: weighted y [32][TC_EPI_LD]
        int* tok = reinterpret_cast<int*>(smem + Sm::epi + 2 * TC_HALF_BYTES);   // token per row [256]
        float* wgt = reinterpret_cast<float*>(tok + 256);                            // weight per row [256]
        __shared__ int epi_abort;
        if (et == 0) epi_abort = 0;
        named_bar(3, 32 * R::EPI);
        int local = 0;
        for (int i = unit; i < n_items; i += n_units, ++local) {
            const Item it = decode_item<PAIR>(a, i, crank);
            const int acc = local & 1;
            const uint32_t accph = (local >> 1) & 1;
            // DOWN: where the item's rows go -- 0 weighted red.add into out, 1 a bf16 row of y_rows,
            // 2 a bf16 row in the sending rank's buffer (peer store)
            const bool shared_item = it.g == a.shared_group;
            const int mode = shared_item ? ((a.y_rows && !a.ymap && !a.meta) ? 1 : 0) : (a.meta ? 2 : (a.y_rows ? 1 : 0));
            // DOWN: thread et looks up the destination and weight of row et while the accumulator
            // fills; it goes to shared memory after the barrier below, when every thread is done with
            // the previous item's lists
            int tk = 0;
            float wk = 0.f;
            if (!GATE_UP && et < it.n) {
                const int rrow = it.row0 + et;
                if (mode == 1) {
                    tk = (a.ymap && !shared_item) ? a.ymap[rrow] : rrow;
                    wk = 1.0f;
                } else if (shared_item) {
                    tk = rrow - a.shared_base;
                    wk = a.sgate[tk];
                } else if (mode == 2) {
                    tk = *reinterpret_cast<volatile const int*>(a.err) == 0 ? a.meta[rrow] : -1;
                    wk = 1.0f;
                } else {
                    const int p = a.pair[rrow];
                    tk = p / a.k;
                    wk = a.wpair[p];
                }
            }
            if (!mbar_wait(&acc_full[acc], accph)) epi_abort = 1;
            named_bar(3, 32 * R::EPI);
            if (epi_abort) break;
            if (!GATE_UP) {   // DOWN: the rows' destinations and weights, strided over the epilogue threads
                if (et < it.n) {
                    tok[et] = tk;
                    wgt[et] = wk;
                }
                for (int rr = et + 32 * R::EPI; rr < it.n; rr += 32 * R::EPI) {
                    const int rrow = it.row0 + rr;
                    int t2;
                    float w2;
                    if (mode == 1) {
                        t2 = (a.ymap && !shared_item) ? a.ymap[rrow] : rrow;
                        w2 = 1.0f;
                    } else if (shared_item) {
                        t2 = rrow - a.shared_base;
                        w2 = a.sgate[t2];
                    } else if (mode == 2) {
                        t2 = *reinterpret_cast<volatile const int*>(a.err) == 0 ? a.meta[rrow] : -1;
                        w2 = 1.0f;
                    } else {
                        const int p = a.pair[rrow];
                        t2 = p / a.k;
                        w2 = a.wpair[p];
                    }
                    tok[rr] = t2;
                    wgt[rr] = w2;
                }
                named_bar(3, 32 * R::EPI);
            }
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(lg * 32) << 16) + acc * 256;
            for (int c0 = 32 * half; c0 < it.n; c0 += 32 * HALVES) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                tmem_ld_wait();
                if (GATE_UP) {
                    // gate warps (rows 0-63) finish columns 0-15, up warps (rows 64-127) columns 16-31
                    if (lg < 2) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) xg[j * 64 + row] = __uint_as_float(v[16 + j]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) xu[j * 64 + row - 64] = __uint_as_float(v[j]);
                    }
                    named_bar(hbar, 128);
                    const int f = row & 63;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float g = lg < 2 ? __uint_as_float(v[j]) : xg[j * 64 + f];
                        const float u = lg < 2 ? xu[j * 64 + f] : __uint_as_float(v[16 + j]);
                        const float h = __fdividef(g, 1.0f + __expf(-g)) * u;
                        hst[(lg < 2 ? j : 16 + j) * 64 + f] = f32_to_bf16_bits(h);
                    }
                    named_bar(hbar, 128);
                    // 32 token rows x 128 B: 4 threads per row, 2 x 16 B each
                    const int j = ht >> 2, part = ht & 3;
                    if (c0 + j < it.n) {
                        const uint4* src = reinterpret_cast<const uint4*>(hst + j * 64 + part * 16);
                        uint4* dst = reinterpret_cast<uint4*>(a.h_out + (size_t)(it.row0 + c0 + j) * a.h_ld +
                                                              it.band * 64 + part * 16);
                        dst[0] = src[0];
                        dst[1] = src[1];
                    }
                    named_bar(hbar, 128);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) ys[j * TC_EPI_LD + row] = __uint_as_float(v[j]) * wgt[c0 + j];
                    named_bar(hbar, 128);
                    // warp w of the half writes tokens 8w..8w+7 of the chunk: 32 lanes x 4 floats = 128 rows
                    const int ew = ht >> 5;
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const int j = ew * 8 + jj;
                        if (c0 + j < it.n) {
                            const float4 y = *reinterpret_cast<const float4*>(ys + j * TC_EPI_LD + lane * 4);
                            if (mode == 0) {
                                red_add_v4(a.out + (size_t)tok[c0 + j] * a.H + it.band * 128 + lane * 4, y);
                            } else if (mode == 2) {
                                const int m = tok[c0 + j];
                                if (m >= 0)
                                    *reinterpret_cast<uint2*>(a.yret[m >> 24] + (size_t)(m & 0xFFFFFF) * a.H +
                                                              it.band * 128 + lane * 4) =
                                        make_uint2(pack_bf16x2(y.x, y.y), pack_bf16x2(y.z, y.w));
                            } else {
                                *reinterpret_cast<uint2*>(a.y_rows + (size_t)tok[c0 + j] * a.H + it.band * 128 + lane * 4) =
                                    make_uint2(pack_bf16x2(y.x, y.y), pack_bf16x2(y.z, y.w));
                            }
                        }
                    }
                    named_bar(hbar, 128);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {   // the warp's TMEM reads are done (on the first CTA's barrier)
                if (PAIR && crank == 1) mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
                else mbar_arrive(&acc_empty[acc]);
            }
        }
        if (epi_abort) {
            fail(a.err, FM_ETIMEOUT);
            atomicExch(&abort_flag, 1);
        }
        if (!GATE_UP && a.meta) __threadfence_system();   // the peer stores land before the rank signals
    }
    tc_fence_before();
    if (PAIR) cluster_sync();   // neither CTA leaves while the other may still signal its barriers
    else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, 512);
        else tmem_dealloc(tmem_base, 512);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// bf16 matrix [rows, cols] with row stride ld elements -> map with a {64, box_rows} box, 128-byte swizzle
// (rows past `rows` read as zeros).
int make_bmap(CUtensorMap* m, const uint16_t* base, int rows, int cols, int ld, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return FM_ECUDA;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d) rows=%d cols=%d ld=%d", (int)r, rows, cols, ld);
        return FM_ECUDA;
    }
    return FM_OK;
}

template <bool GATE_UP, bool PAIR>
static cudaError_t launch_tc_variant(const CUtensorMap& bmap, const CUtensorMap& bmap_big, const TcArgs& a, int grid,
                                     int sm, cudaStream_t st) {
    if (cudaError_t e = raise_smem_limit((const void*)expert_tc_kernel<GATE_UP, PAIR>, sm)) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(TcRoles<GATE_UP>::THREADS);
    cfg.dynamicSmemBytes = sm;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = PAIR ? 2 : 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, expert_tc_kernel<GATE_UP, PAIR>, bmap, bmap_big, a);
}

int launch_expert_tc(bool gate_up, const TcLaunch& L, cudaStream_t st) {
    if (L.max_items <= 0) return FM_OK;
    CUtensorMap bmap, bmap_big;
    if (int rc = make_bmap(&bmap, L.act, L.act_rows, L.act_cols, L.act_ld, TC_BOX_ROWS)) return rc;
    if (int rc = make_bmap(&bmap_big, L.act, L.act_rows, L.act_cols, L.act_ld, TC_BOX_BIG)) return rc;
    TcArgs a{};
    a.list = L.list;
    a.w_routed = L.w_routed;
    a.w_routed_stride = L.w_routed_stride;
    a.w_shared = L.w_shared;
    a.shared_group = L.shared_group;
    a.K_routed = L.K_routed;
    a.K_shared = L.K_shared;
    a.h_out = L.h_out;
    a.h_ld = L.h_ld;
    a.out = L.out;
    a.H = L.H;
    a.pair = L.pair;
    a.wpair = L.wpair;
    a.k = L.k;
    a.shared_base = L.shared_base;
    a.sgate = L.sgate;
    a.y_rows = L.y_rows;
    a.ymap = L.ymap;
    a.meta = L.meta;
    for (int i = 0; i < kMaxRanks; ++i) a.yret[i] = L.yret[i];
    a.err = L.err;
    int sms = device_sm_count();
    if (L.max_ctas > 0 && L.max_ctas < sms) sms = L.max_ctas;
    const int sm_single = gate_up ? TcSmem<true, false>::total : TcSmem<false, false>::total;
    const int sm_pair = gate_up ? TcSmem<true, true>::total : TcSmem<false, true>::total;
    cudaError_t e;
    if (L.cta_pair) {
        // one pair per two SMs; items are band pairs
        const int pairs = L.max_items < sms / 2 ? L.max_items : sms / 2;
        e = gate_up ? launch_tc_variant<true, true>(bmap, bmap_big, a, 2 * pairs, sm_pair, st)
                    : launch_tc_variant<false, true>(bmap, bmap_big, a, 2 * pairs, sm_pair, st);
    } else {
        const int grid = L.max_items < sms ? L.max_items : sms;
        e = gate_up ? launch_tc_variant<true, false>(bmap, bmap_big, a, grid, sm_single, st)
                    : launch_tc_variant<false, false>(bmap, bmap_big, a, grid, sm_single, st);
    }
    if (e != cudaSuccess) {
        note_launch();
        return cuda_status(e, gate_up ? "expert_tc<gate_up>" : "expert_tc<down>");
    }
    FM_LAUNCH_CHECK(gate_up ? "expert_tc<gate_up>" : "expert_tc<down>");
    return FM_OK;
}

}  // namespace fm
