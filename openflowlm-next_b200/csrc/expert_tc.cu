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
//               the raw tile (two GGUF blocks) into 64 bf16 values in the 128-byte-swizzled K-major
//               layout the MMA reads (w = q*d + m in f32 with the fp16 d, m widened exactly, paired
//               f32x2 FMAs, rounded once to bf16);
//   warps 10-   epilogue (gate_up 4 warps; down 8 in two halves taking alternate 32-token chunks),
//               overlapped with the next item's main loop through the second accumulator:
//               GATE_UP  rows 0-63 of a gate_up tile are gate rows, rows 64-127 the up rows of the same
//                        64 features: h = bf16(silu(g) * u) -> the sorted h matrix (the reference's
//                        SwiGLU, designs/moe_batch/moe_batch.h:181-202, h rounded to bf16);
//               DOWN     out[token][row] += w * y (the weighted scatter of core.cpp:5236-5255, routing
//                        weight or shared-expert gate per row): the weighted 32-token chunk is staged
//                        in shared memory, then each warp adds 8 token rows with red.global.add.v4.f32;
//                        or unweighted f32 y rows for a fixed-order combine after the kernel; or
//                        unweighted bf16 y rows (expert parallel: in the received order, or straight
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
constexpr int TC_BN = kTcItemRows;         // max tokens per work item (MMA N)
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
// Both: 4 activation stages of 256 rows (128 KB). Two dequantiser groups take alternate slabs, so with 4
// A stages each group has a second stage to fill while the tensor core still reads its first.
// Shared-memory bandwidth, not the tensor pipe, bounds the main loop: per 64-K slab of a 256-token item
// the activation stage is written by TMA and read by the MMAs (32 KB each way), the A stage written by
// the dequantisers and read by the MMAs (16 KB each way) and the raw tile written and read (5 KB each),
// about 210 bytes per clock at the MMAs' full rate against the SM's 128.
template <bool GATE_UP>
struct TcSmem {
    static constexpr int SA = GATE_UP ? 4 : 2;
    static constexpr int SB = 4;
    static constexpr int SR = GATE_UP ? 4 : 6;    // raw weight tiles in flight (streamed from HBM)
    // Slabs per pipeline stage: the MMA issuer waits, issues and commits once per stage, so the hand-off
    // between the roles (barrier waits, commits) is paid once per KS slabs' MMAs. gate_up takes two 64-K
    // slabs per stage (8 MMAs), one per dequantiser group; down (K = 512, 8 slabs) keeps one.
    static constexpr int KS = GATE_UP ? 2 : 1;
    static constexpr int SAQ = SA / KS, SBQ = SB / KS;   // stages of the A and activation rings
    static constexpr int B_STAGE = TC_B_BYTES;
    static constexpr int EPI = GATE_UP ? 3 * 16 * 64 * 4 : TC_EPI_BYTES;
    // offsets from the 1024-aligned dynamic smem base
    static constexpr int a = 0;
    static constexpr int b = a + SA * TC_A_BYTES;
    static constexpr int raw = b + SB * B_STAGE;
    static constexpr int epi = raw + SR * kTileBytes;
    static constexpr int bars = epi + EPI;
    // raw, activation, A and accumulator rings + drain
    static constexpr int nbars = 2 * SR + 2 * SBQ + 2 * SAQ + 4 + 1;
    static constexpr int tmem = bars + nbars * 8;
    static constexpr int total = tmem + 16 + 1024;   // + alignment slack
};
static_assert(TcSmem<true>::total <= 232448 && TcSmem<false>::total <= 232448, "shared memory per CTA");

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
    // DOWN, f32 row mode (the fixed-order combine): every row's y, unweighted f32, goes to y_f32[r] (routed
    // and shared rows alike); a combine kernel then sums each token in ascending expert order
    float* y_f32;
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

// (x, y) * (D, D) + (C, C) as one packed f32x2 FMA.
__device__ __forceinline__ float2 fma2(float2 x, float2 D, float2 C) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(r)
        : "l"(*reinterpret_cast<unsigned long long*>(&x)), "l"(*reinterpret_cast<unsigned long long*>(&D)),
          "l"(*reinterpret_cast<unsigned long long*>(&C)));
    return *reinterpret_cast<float2*>(&r);
}

// Four codes (bytes 0-3 of t) -> two bf16x2 words of q*d + m: (byte 0, byte 1) and (byte 2, byte 3).
__device__ __forceinline__ uint2 deq4(uint32_t t, float2 D, float2 C) {
    const float2 a = fma2(make_float2(code_f(t, 0x7044), code_f(t, 0x7144)), D, C);
    const float2 b = fma2(make_float2(code_f(t, 0x7244), code_f(t, 0x7344)), D, C);
    return make_uint2(pack_bf16x2(a.x, a.y), pack_bf16x2(b.x, b.y));
}

// One GGUF block in the tile's word order (word c = bytes b(2c), b(2c+1), b(2c+8), b(2c+9); byte j holds
// value j in its low nibble, value j + 16 in its high one) -> its 16 bf16x2 words in K order (word j =
// values 2j, 2j+1) at out[0..15].
__device__ __forceinline__ void deq_block(uint4 n, float d, float m, uint32_t* out) {
    const float2 D = make_float2(256.0f * d, 256.0f * d);
    const float cm = fmaf(-128.0f, d, m);
    const float2 C = make_float2(cm, cm);
    const uint32_t w[4] = {n.x, n.y, n.z, n.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint2 lo = deq4(w[c] & 0x0F0F0F0Fu, D, C);          // values 2c, 2c+1 | 2c+8, 2c+9
        const uint2 hi = deq4((w[c] >> 4) & 0x0F0F0F0Fu, D, C);   // values 2c+16, 2c+17 | 2c+24, 2c+25
        out[c] = lo.x;
        out[c + 4] = lo.y;
        out[c + 8] = hi.x;
        out[c + 12] = hi.y;
    }
}

struct Item {
    int g, band, row0, n, slabs;
    const uint8_t* w;
};

__device__ __forceinline__ Item decode_item(const TcArgs& a, int i) {
    const int4 it = reinterpret_cast<const int4*>(a.list + 4)[i];
    Item r;
    r.g = it.x;
    r.band = it.y;
    r.row0 = it.z;
    r.n = it.w;
    const bool sh = r.g == a.shared_group;
    const int K = sh ? a.K_shared : a.K_routed;
    r.slabs = K / kTileK;
    const uint8_t* base = sh ? a.w_shared : a.w_routed + (size_t)r.g * a.w_routed_stride;
    r.w = base + (size_t)r.band * r.slabs * kTileBytes;
    return r;
}

template <bool GATE_UP>
__global__ void __launch_bounds__(TcRoles<GATE_UP>::THREADS, 1) expert_tc_kernel(const __grid_constant__ CUtensorMap bmap,
                                                                  const __grid_constant__ CUtensorMap bmap_big, TcArgs a) {
    using R = TcRoles<GATE_UP>;
    using Sm = TcSmem<GATE_UP>;
    constexpr int SR = Sm::SR, B_STAGE = Sm::B_STAGE, KS = Sm::KS, SAQ = Sm::SAQ, SBQ = Sm::SBQ;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Sm::bars);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = raw_full + SR;
    uint64_t* b_full = raw_empty + SR;           // per stage of KS slabs
    uint64_t* b_empty = b_full + SBQ;
    uint64_t* a_full = b_empty + SBQ;
    uint64_t* a_empty = a_full + SAQ;
    uint64_t* acc_full = a_empty + SAQ;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;             // the MMA issuer's last commit
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Sm::tmem);
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = a.list[0];
    const int unit = (int)blockIdx.x, n_units = (int)gridDim.x;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        // a dequantiser group (4 warps, 128 threads) consumes a raw tile and fills an A stage
        for (int i = 0; i < SR; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], 128); }
        for (int i = 0; i < SBQ; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
        // arrivals are per warp: the dequantiser warps filling a stage (4 per slab) / 4 or 8 epilogue warps
        for (int i = 0; i < SAQ; ++i) { mbar_init(&a_full[i], 4 * KS); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], R::EPI); }
        mbar_init(drain, 1);
        mbar_fence_init();
        prefetch_tmap(&bmap);
        prefetch_tmap(&bmap_big);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0 || warp == R::BWARP) {
        // ------------------------------------------------------------ producers (lane 0 of each)
        // warp 0: the raw weight tiles (streamed from HBM, SR deep); warp R::BWARP: the activation
        // rows (TMA, SB deep). Separate threads, so the weight stream runs ahead of the activations.
        const bool weights = warp == 0;
        if (lane == 0) {
            const int S = weights ? SR : SBQ;
            const int KU = weights ? 1 : KS;   // slabs per fill: one raw tile, or a stage of activations
            uint64_t* full = weights ? raw_full : b_full;
            uint64_t* empty = weights ? raw_empty : b_empty;
            int st = 0;
            uint32_t ph = 0, issued = 0;   // bit i: slot i has a fill in flight or landed
            bool ok = true;
            for (int i = unit; i < n_items && ok; i += n_units) {
                const Item it = decode_item(a, i);
                const int nhalf = it.n;
                const int rbase = it.row0;
                // whole 128-row boxes, then 32-row boxes for the rest
                const int nbig = nhalf / TC_BOX_BIG;
                const int nsmall = (nhalf - nbig * TC_BOX_BIG + TC_BOX_ROWS - 1) / TC_BOX_ROWS;
                const int rows_loaded = nbig * TC_BOX_BIG + nsmall * TC_BOX_ROWS;
                for (int s = 0; s < it.slabs; s += KU) {
                    if (!mbar_wait(&empty[st], ph ^ 1)) { ok = false; break; }
                    if (weights) {
                        mbar_expect_tx(&raw_full[st], kTileBytes);
                        bulk_load(smem + Sm::raw + st * kTileBytes, it.w + (size_t)s * kTileBytes, kTileBytes, &raw_full[st]);
                        issued |= 1u << st;
                    } else {
                        const int ns = min(KU, it.slabs - s);   // slabs in this stage
                        mbar_expect_tx(&b_full[st], ns * rows_loaded * 128);
                        for (int h = 0; h < ns; ++h)
                            for (int j = 0; j < nbig + nsmall; ++j) {
                                const bool big = j < nbig;
                                const int r0 = big ? j * TC_BOX_BIG : nbig * TC_BOX_BIG + (j - nbig) * TC_BOX_ROWS;
                                const CUtensorMap* map = big ? &bmap_big : &bmap;
                                uint8_t* dst = smem + Sm::b + (st * KS + h) * B_STAGE + r0 * 128;
                                tma_load_2d(dst, map, (s + h) * kTileK, rbase + r0, &b_full[st]);
                            }
                        issued |= 1u << st;
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
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int as = 0, bs = 0;
            uint32_t aph = 0, bph = 0;
            bool ok = true, issued = false;
            int local = 0;
            for (int i = unit; i < n_items && ok; i += n_units, ++local) {
                const Item it = decode_item(a, i);
                const int acc = local & 1;
                const uint32_t accph = (local >> 1) & 1;
                if (!mbar_wait(&acc_empty[acc], accph ^ 1)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * 256;
                const uint32_t idesc = idesc_bf16(128, (it.n + 15) & ~15);
                for (int s = 0; s < it.slabs; s += KS) {
                    if (!mbar_wait(&a_full[as], aph) || !mbar_wait(&b_full[bs], bph)) { ok = false; break; }
                    tc_fence_after();
                    const int ns = min(KS, it.slabs - s);
                    for (int h = 0; h < ns; ++h) {
                        const uint32_t sa = smem_u32(smem + Sm::a + (as * KS + h) * TC_A_BYTES);
                        const uint32_t sb = smem_u32(smem + Sm::b + (bs * KS + h) * B_STAGE);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc_mma_f16(d_tmem, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + kk * 32), idesc,
                                       (s > 0 || h > 0 || kk > 0) ? 1u : 0u);
                    }
                    issued = true;
                    tc_commit(&a_empty[as]);
                    tc_commit(&b_empty[bs]);
                    if (++as == SAQ) { as = 0; aph ^= 1; }
                    if (++bs == SBQ) { bs = 0; bph ^= 1; }
                }
                if (!ok) break;
                tc_commit(&acc_full[acc]);
            }
            if (!ok) {
                fail(a.err, FM_ETIMEOUT);
                atomicExch(&abort_flag, 1);
            }
            // every MMA of this CTA (and its commits' arrivals) done before the CTA may exit
            if (issued) {
                tc_commit(drain);
                mbar_wait(drain, 0);
            }
        }
    } else if (warp < R::EPI0) {
        // ------------------------------------------------------------ dequantisers
        // Groups of 4 warps; thread t of a group rebuilds row t of a tile (both 32-value blocks). With two
        // slabs per stage (gate_up) group g takes slab g of every stage, so both groups fill a stage at
        // once; with one (down) the groups take alternate stages. Either way two slabs are dequantised at
        // once (the per-slab chain of barrier, shared loads and stores is latency-bound).
        constexpr int NG = R::DQ / 4;
        const int t = threadIdx.x - 64;
        const int grp = t >> 7;
        const int r = t & 127;
        const int h = KS == NG ? grp : 0;   // this group's slab within a stage
        bool ok = true;
        int qc = 0, scb = 0;   // running stage index over this CTA's items; slabs of its earlier items
        for (int i = unit; i < n_items && ok; i += n_units) {
            const Item it = decode_item(a, i);
            const int nst = (it.slabs + KS - 1) / KS;
            for (int q = 0; q < nst; ++q, ++qc) {
                if (KS == 1 && qc % NG != grp) continue;
                const int s = q * KS + h;
                const bool has = s < it.slabs;   // the last stage of an odd slab count has one slab
                const int as = qc % SAQ;
                const uint32_t aph = (qc / SAQ) & 1;
                uint32_t wv[32];   // the row's 64 values in K order: 16-byte chunk c = words 4c..4c+3
                if (has) {
                    const int rs = (scb + s) % SR;
                    const uint32_t rph = ((scb + s) / SR) & 1;
                    if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[rs], rph))) { ok = false; break; }
                    const uint32_t raw = smem_u32(smem + Sm::raw + rs * kTileBytes);
                    const uint4 n0 = lds128(raw + r * 32);
                    const uint4 n1 = lds128(raw + r * 32 + 16);
                    const uint2 sc2 = lds64(raw + kTileNibBytes + r * 8);
                    const float d0 = __half2float(__ushort_as_half((unsigned short)(sc2.x & 0xFFFF)));
                    const float m0 = __half2float(__ushort_as_half((unsigned short)(sc2.x >> 16)));
                    const float d1 = __half2float(__ushort_as_half((unsigned short)(sc2.y & 0xFFFF)));
                    const float m1 = __half2float(__ushort_as_half((unsigned short)(sc2.y >> 16)));
                    deq_block(n0, d0, m0, wv);
                    deq_block(n1, d1, m1, wv + 16);
                    // The raw slot goes back to the weight producer, whose next bulk copy (async proxy)
                    // overwrites it, only after this thread's loads from it have delivered their values (the
                    // dequantised words depend on them) and a proxy fence: releasing it right after issuing
                    // the loads let the copy land under loads still in flight on B200 (wrong weights for a
                    // slab, intermittently).
                    fence_proxy_async_smem();
                    mbar_arrive(&raw_empty[rs]);
                }
                if (!__all_sync(0xffffffffu, mbar_wait(&a_empty[as], aph ^ 1))) { ok = false; break; }
                if (has) {
                    const uint32_t arow = smem_u32(smem + Sm::a + (as * KS + h) * TC_A_BYTES + r * 128);
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        sts128(arow + ((c ^ (r & 7)) << 4),
                               make_uint4(wv[4 * c], wv[4 * c + 1], wv[4 * c + 2], wv[4 * c + 3]));
                    fence_proxy_async_smem();
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[as]);   // the warp's 32 rows are in place (or absent)
            }
            scb += it.slabs;
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
            const Item it = decode_item(a, i);
            const int acc = local & 1;
            const uint32_t accph = (local >> 1) & 1;
            // DOWN: where the item's rows go -- 0 weighted red.add into out, 1 a bf16 row of y_rows,
            // 2 a bf16 row in the sending rank's buffer (peer store)
            const bool shared_item = it.g == a.shared_group;
            const int mode = a.y_f32 ? 3
                             : shared_item ? ((a.y_rows && !a.ymap && !a.meta) ? 1 : 0) : (a.meta ? 2 : (a.y_rows ? 1 : 0));
            // DOWN: thread et looks up the destination and weight of row et while the accumulator
            // fills; it goes to shared memory after the barrier below, when every thread is done with
            // the previous item's lists
            int tk = 0;
            float wk = 0.f;
            if (!GATE_UP && et < it.n) {
                const int rrow = it.row0 + et;
                if (mode == 1 || mode == 3) {
                    tk = (mode == 1 && a.ymap && !shared_item) ? a.ymap[rrow] : rrow;
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
                    if (mode == 1 || mode == 3) {
                        t2 = (mode == 1 && a.ymap && !shared_item) ? a.ymap[rrow] : rrow;
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
                            } else if (mode == 3) {
                                *reinterpret_cast<float4*>(a.y_f32 + (size_t)tok[c0 + j] * a.H + it.band * 128 + lane * 4) = y;
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
            if (lane == 0) mbar_arrive(&acc_empty[acc]);   // the warp's TMEM reads are done
        }
        if (epi_abort) {
            fail(a.err, FM_ETIMEOUT);
            atomicExch(&abort_flag, 1);
        }
        if (!GATE_UP && a.meta) __threadfence_system();   // the peer stores land before the rank signals
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
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

template <bool GATE_UP>
static cudaError_t launch_tc_variant(const CUtensorMap& bmap, const CUtensorMap& bmap_big, const TcArgs& a, int grid,
                                     cudaStream_t st) {
    const int sm = TcSmem<GATE_UP>::total;
    if (cudaError_t e = raise_smem_limit((const void*)expert_tc_kernel<GATE_UP>, sm)) return e;
    expert_tc_kernel<GATE_UP><<<grid, TcRoles<GATE_UP>::THREADS, sm, st>>>(bmap, bmap_big, a);
    return cudaGetLastError();
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
    a.y_f32 = L.y_f32;
    a.meta = L.meta;
    for (int i = 0; i < kMaxRanks; ++i) a.yret[i] = L.yret[i];
    a.err = L.err;
    int sms = device_sm_count();
    if (L.max_ctas > 0 && L.max_ctas < sms) sms = L.max_ctas;
    const int grid = L.max_items < sms ? L.max_items : sms;
    const cudaError_t e = gate_up ? launch_tc_variant<true>(bmap, bmap_big, a, grid, st)
                                  : launch_tc_variant<false>(bmap, bmap_big, a, grid, st);
    if (e != cudaSuccess) {
        note_launch();
        return cuda_status(e, gate_up ? "expert_tc<gate_up>" : "expert_tc<down>");
    }
    FM_LAUNCH_CHECK(gate_up ? "expert_tc<gate_up>" : "expert_tc<down>");
    return FM_OK;
}

}  // namespace fm
