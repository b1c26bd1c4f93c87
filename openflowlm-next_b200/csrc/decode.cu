// Decode-size path (T <= 32 tokens): small-T router logits, single-CTA dispatch that also builds the
// GEMV work lists, and the bandwidth-bound grouped Q4_1 GEMV.
//
// GEMV: each work item is (group, 128-row band, up to 8 sorted rows, K chunk). One CTA per SM: a
// producer warp keeps 24 weight tiles (120 KB) of bulk copies in flight and double-buffers each item's
// bf16 activation rows; 16 consumer warps in two groups take alternate slab pairs, each warp 32 rows
// of the band and one of the slab's two 32-value blocks. The tensor core multiplies the
// raw codes, never dequantised weights: the A operand is 128 + q as bf16 (exact; one byte permute per
// two codes, one 32-bit load per fragment thanks to the tile's fragment byte order), the B operand the
// bf16 activations, so per 32-value block C = sum (128 + q) x exactly in f32, and the block's exact fp16
// scale d and min m are applied after the MMA:
//   y += d * C + (m - 128 d) * X,   X = sum of the block's activations,
// i.e. the oracle's exact dequantisation (q4_1_pack.py:104-109) with only f32 roundings. K is split
// into up to 4 chunks when fewer than half the SMs would have work; the last CTA to finish a (group,
// band, rows) item reduces the chunks in order.
//   GATE_UP: tile rows 0-63 gate, 64-127 up of 64 features -> h = bf16(silu(g) * u) (moe_batch.h:181-202)
//   DOWN:    y rows (f32) -> combine_kernel sums each token's experts in ascending order.
#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace fm {

// ------------------------------------------------------------------ single-CTA dispatch + GEMV lists
// Pairs P <= 1024. Same results as dispatch_{hist,scan,scatter} (stable, token-then-slot order within an
// expert), plus the GEMV work lists: items (g | band << 16, row0, n | kc << 16, slot), list[0] = count,
// list[1] = chunks per item row group.
constexpr int kGemvRows = 8;        // sorted rows (tokens) per GEMV item
constexpr int kDispSmallThreads = 1024;

// Block-wide (1024 threads) exclusive scan / sum of one int per thread; sh holds 32 ints.
__device__ int block_exclusive_scan_1024(int v, int* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) sh[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int s = sh[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        sh[lane] = s;
    }
    __syncthreads();
    const int r = (warp ? sh[warp - 1] : 0) + x - v;
    __syncthreads();
    return r;
}

__device__ int block_sum_1024(int v, int* sh) {
    const int ex = block_exclusive_scan_1024(v, sh);
    __shared__ int tot;
    if (threadIdx.x == 1023) tot = ex + v;
    __syncthreads();
    const int t = tot;
    __syncthreads();
    return t;
}

// K split per item group: only when fewer than half the SMs would otherwise have work (a split costs a
// round trip through the partial buffer and a completion counter).
__device__ int choose_chunks(int base_items, int slabs) {
    int kc = base_items >= 74 ? 1 : base_items >= 37 ? 2 : 4;
    while (kc > 1 && slabs % kc) kc >>= 1;
    return kc;
}

__global__ void __launch_bounds__(kDispSmallThreads) dispatch_small_kernel(
    const int32_t* __restrict__ idx, int P, int e_begin, int e_local, int shared_base, int shared_rows,
    int* __restrict__ counts, int* __restrict__ offsets, int* __restrict__ pos, int* __restrict__ pair,
    int* __restrict__ gu_list, int gu_bands, int gu_bands_shared, int gu_slabs, int* __restrict__ dn_list, int dn_bands,
    int dn_slabs, int dn_slabs_shared, int* __restrict__ err) {
    extern __shared__ int sm[];
    int* cnt = sm;                                  // [e_local]
    int* wcnt = cnt + e_local;                      // [32][e_local]
    int* scan_sh = wcnt + 32 * e_local;             // [32]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < e_local; e += blockDim.x) {
        cnt[e] = 0;
        for (int w = 0; w < 32; ++w) wcnt[w * e_local + e] = 0;
    }
    __syncthreads();
    // one pair per thread (P <= 1024): local expert or -1
    const int p = threadIdx.x;
    int e = -1;
    if (p < P) {
        e = idx[p] - e_begin;
        if (e < 0 || e >= e_local) {
            atomicAdd(err, 1);
            e = -1;
        }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wcnt[warp * e_local + e] = __popc(peers);
    __syncthreads();
    // per expert: prefix over warps (in place) and total
    for (int x = threadIdx.x; x < e_local; x += blockDim.x) {
        int s = 0;
        for (int w = 0; w < 32; ++w) {
            const int v = wcnt[w * e_local + x];
            wcnt[w * e_local + x] = s;
            s += v;
        }
        cnt[x] = s;
    }
    __syncthreads();
    // exclusive scan of counts over experts (e_local <= 1024)
    {
        const int v = threadIdx.x < e_local ? cnt[threadIdx.x] : 0;
        int xs = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, xs, o);
            if (lane >= o) xs += y;
        }
        if (lane == 31) scan_sh[warp] = xs;
        __syncthreads();
        if (warp == 0) {
            int s = scan_sh[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            scan_sh[lane] = s;
        }
        __syncthreads();
        const int ex = (warp ? scan_sh[warp - 1] : 0) + xs - v;
        if (threadIdx.x < e_local) {
            counts[threadIdx.x] = v;
            offsets[threadIdx.x] = ex;
        }
        if (threadIdx.x == 0) {
            counts[e_local] = shared_rows;
            offsets[e_local] = scan_sh[31];
            offsets[e_local + 1] = shared_base;
        }
        __syncthreads();
    }
    if (e >= 0) {
        const int b = offsets[e] + wcnt[warp * e_local + e] + rank;
        pos[p] = b;
        pair[b] = p;
    } else if (p < P) {
        pos[p] = -1;
    }
    // GEMV work lists: thread g emits group g's items (G <= 1024 groups)
    const int G = e_local + (shared_rows > 0 ? 1 : 0);
    const int gi = threadIdx.x;
    int c_g = 0, r0_g = 0, bands_g = 0, tt = 0;
    if (gi < G) {
        c_g = gi < e_local ? counts[gi] : shared_rows;
        r0_g = gi < e_local ? offsets[gi] : shared_base;
        bands_g = gi < e_local ? gu_bands : gu_bands_shared;
        tt = (c_g + kGemvRows - 1) / kGemvRows;
    }
    const int bgu = tt * bands_g, bdn = tt * dn_bands;
    const int tot_gu = block_sum_1024(bgu, scan_sh), tot_dn = block_sum_1024(bdn, scan_sh);
    const int kc_gu = choose_chunks(tot_gu, gu_slabs);
    int kc_dn = choose_chunks(tot_dn, dn_slabs);
    if (shared_rows > 0) while (kc_dn > 1 && dn_slabs_shared % kc_dn) kc_dn >>= 1;
    const int slot_gu = block_exclusive_scan_1024(bgu, scan_sh), slot_dn = block_exclusive_scan_1024(bdn, scan_sh);
    if (gi < G && c_g > 0) {
        int ngu = slot_gu * kc_gu, ndn = slot_dn * kc_dn, sgu = slot_gu, sdn = slot_dn;
        for (int r = 0; r < c_g; r += kGemvRows) {
            const int n = min(kGemvRows, c_g - r);
            for (int b = 0; b < bands_g; ++b, ++sgu)
                for (int kc = 0; kc < kc_gu; ++kc, ++ngu)
                    reinterpret_cast<int4*>(gu_list + 4)[ngu] = make_int4(gi | (b << 16), r0_g + r, n | (kc << 16), sgu);
            for (int b = 0; b < dn_bands; ++b, ++sdn)
                for (int kc = 0; kc < kc_dn; ++kc, ++ndn)
                    reinterpret_cast<int4*>(dn_list + 4)[ndn] = make_int4(gi | (b << 16), r0_g + r, n | (kc << 16), sdn);
        }
    }
    if (threadIdx.x == 0) {
        gu_list[0] = tot_gu * kc_gu;
        gu_list[1] = kc_gu;
        dn_list[0] = tot_dn * kc_dn;
        dn_list[1] = kc_dn;
    }
}

// ------------------------------------------------------------------ grouped Q4_1 GEMV
struct GemvArgs {
    const int* list;
    const uint8_t* w_routed;
    size_t w_routed_stride;
    const uint8_t* w_shared;
    int shared_group;
    int K_routed, K_shared;
    // bf16 activations: GATE_UP the token rows (x [T, H]), DOWN the sorted h rows ([rows, Fmax])
    const uint16_t* act;
    int act_ld;
    const int* pair;          // GATE_UP: sorted row -> pair id (routed rows)
    int k;
    int shared_base;
    // outputs
    float* part;              // [4][rows][out_cols] f32 partial sums (K split)
    int part_rows;
    int* done;                // completion counters per item slot (zeroed per call)
    uint16_t* h_out;          // GATE_UP final: bf16 h [rows, h_ld]
    int h_ld;
    int F_routed, F_shared;   // GATE_UP: features per matrix
    float* y_out;             // DOWN final: f32 [rows, H]
    int H;
    int* err;                 // FM_ETIMEOUT when a bounded wait gives up
};

constexpr int GV_GWARPS = 8;                          // warps of a consumer group: 32 tile rows x one of 2 blocks
constexpr int GV_GROUPS = 2;                          // groups take alternate slab pairs of an item
constexpr int GV_CONSUMERS = GV_GWARPS * GV_GROUPS;   // consumer warps
constexpr int GV_THREADS = 32 * (GV_CONSUMERS + 1);   // + one producer warp
constexpr int GV_MAX_K = 2048;                        // activation K per item (one chunk)
constexpr int GV_WSTAGES = 24;                        // weight tiles in flight per CTA (120 KB)
constexpr int GV_XLD = GV_MAX_K + 8;                  // bf16 row of the staged activations (bank spread)
constexpr int GV_ACT_BYTES = kGemvRows * GV_XLD * 2;  // bf16 rows of one item

struct GvSmem {
    static constexpr int w = 0;
    static constexpr int act = w + GV_WSTAGES * kTileBytes;
    static constexpr int tab = act + 2 * GV_ACT_BYTES;                 // [8 warps][2 slabs][32] (d, m - 128 d)
    static constexpr int xch = tab + GV_CONSUMERS * 64 * 8;            // [128][8] f32 (block-1 partials, up rows)
    static constexpr int xch2 = xch + 128 * kGemvRows * 4;             // [2][128][8] f32 (group-1 partials)
    static constexpr int bars = xch2 + 2 * 128 * kGemvRows * 4;
    static constexpr int total = bars + (2 * GV_WSTAGES + 4) * 8 + 128;
};

__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One 32-value block (blk) of NS consecutive slabs (their tiles in tiles[]) for the warp's 32 rows
// (two m16 tiles) and 8 token columns: acc[tile] (C fragments of m16n8) += the exact Q4_1 products.
// xs: staged activations [8][GV_XLD] from the chunk start; tab: this warp's (d, m - 128 d) per row and
// slab. The block sums X come from the tensor core too: an MMA with an all-ones A operand, shared by
// both row tiles. The NS slabs are independent chains, interleaved by the compiler.
template <int NS>
__device__ __forceinline__ void gv_blocks(const uint8_t* const* tiles, const uint16_t* xs, float2* tab, int s0, int blk,
                                          int rg, int lane, float (*acc)[4]) {
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int j = 0; j < NS; ++j) {   // lane r converts the scale pair of row 32 rg + r of this block
        const uint32_t sc = *reinterpret_cast<const uint32_t*>(tiles[j] + kTileNibBytes + (rg * 32 + lane) * 8 + blk * 4);
        const float d = __half2float(__ushort_as_half((unsigned short)(sc & 0xFFFF)));
        const float m = __half2float(__ushort_as_half((unsigned short)(sc >> 16)));
        tab[j * 32 + lane] = make_float2(d, fmaf(-128.f, d, m));
    }
    uint32_t u[NS][4];   // rows g, g+8, g+16, g+24 of the warp's 32
#pragma unroll
    for (int j = 0; j < NS; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r)
            u[j][r] = *reinterpret_cast<const uint32_t*>(tiles[j] + (rg * 32 + g + 8 * r) * 32 + blk * 16 + c * 4);
    float cb[NS][2][4] = {}, cx[NS][4] = {};
    const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
#pragma unroll
    for (int hi = 0; hi < 2; ++hi) {
#pragma unroll
        for (int j = 0; j < NS; ++j) {
            const uint16_t* xr = xs + g * GV_XLD + (s0 + j) * kTileK + blk * 32 + hi * 16 + 2 * c;
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr), b1 = *reinterpret_cast<const uint32_t*>(xr + 8);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const uint32_t ta = (u[j][2 * mt] >> (4 * hi)) & 0x0F0F0F0Fu, tb = (u[j][2 * mt + 1] >> (4 * hi)) & 0x0F0F0F0Fu;
                uint32_t af[4];
                af[0] = __byte_perm(ta, 0x4343u, 0x5140);   // 128 + q of values 2c, 2c+1
                af[1] = __byte_perm(tb, 0x4343u, 0x5140);
                af[2] = __byte_perm(ta, 0x4343u, 0x5342);   // values 2c+8, 2c+9
                af[3] = __byte_perm(tb, 0x4343u, 0x5342);
                mma_bf16(cb[j][mt], af, b0, b1);
            }
            mma_bf16(cx[j], ones, b0, b1);
        }
    }
    __syncwarp();
    // cx[0] / cx[1]: sum of the block's activations of tokens 2c / 2c+1 (every row alike)
#pragma unroll
    for (int j = 0; j < NS; ++j)
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            const float2 sa = tab[j * 32 + 16 * mt + g], sb = tab[j * 32 + 16 * mt + g + 8];
            acc[mt][0] = fmaf(sa.x, cb[j][mt][0], fmaf(sa.y, cx[j][0], acc[mt][0]));
            acc[mt][1] = fmaf(sa.x, cb[j][mt][1], fmaf(sa.y, cx[j][1], acc[mt][1]));
            acc[mt][2] = fmaf(sb.x, cb[j][mt][2], fmaf(sb.y, cx[j][0], acc[mt][2]));
            acc[mt][3] = fmaf(sb.x, cb[j][mt][3], fmaf(sb.y, cx[j][1], acc[mt][3]));
        }
    __syncwarp();
}

struct GvItem {
    int grp, bnd, row0, n, kc, slot, slabs, s0, kn;
    bool sh;
    const uint8_t* wband;
};

__device__ __forceinline__ GvItem gv_decode(const GemvArgs& a, int i, int KC) {
    const int4 it = reinterpret_cast<const int4*>(a.list + 4)[i];
    GvItem r;
    r.grp = it.x & 0xFFFF;
    r.bnd = it.x >> 16;
    r.row0 = it.y;
    r.n = it.z & 0xFFFF;
    r.kc = it.z >> 16;
    r.slot = it.w;
    r.sh = r.grp == a.shared_group;
    const int K = r.sh ? a.K_shared : a.K_routed;
    r.slabs = K / kTileK / KC;
    r.s0 = r.kc * r.slabs;
    r.kn = r.slabs * kTileK;
    r.wband = (r.sh ? a.w_shared : a.w_routed + (size_t)r.grp * a.w_routed_stride) + (size_t)r.bnd * (K / kTileK) * kTileBytes;
    return r;
}

template <bool GATE_UP>
__global__ void __launch_bounds__(GV_THREADS, 1) gemv_kernel(GemvArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint64_t* w_full = reinterpret_cast<uint64_t*>(smem + GvSmem::bars);
    uint64_t* w_empty = w_full + GV_WSTAGES;
    uint64_t* act_full = w_empty + GV_WSTAGES;
    uint64_t* act_empty = act_full + 2;
    float* xch = reinterpret_cast<float*>(smem + GvSmem::xch);
    __shared__ int s_last, s_abort;   // s_abort: consumer warps only
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = a.list[0], KC = a.list[1];
    if (threadIdx.x == 0) {
        for (int i = 0; i < GV_WSTAGES; ++i) { mbar_init(&w_full[i], 1); mbar_init(&w_empty[i], GV_GWARPS); }
        for (int i = 0; i < 2; ++i) { mbar_init(&act_full[i], 1); mbar_init(&act_empty[i], GV_CONSUMERS); }
        s_abort = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == GV_CONSUMERS) {
        // ------------------------------------------------------------ producer warp
        int ws = 0, ab = 0;
        uint32_t wph = 0, aph = 0;
        bool ok = true;
        for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
            const GvItem it = gv_decode(a, i, KC);
            // the item's activations: int16 rows by bulk copy, block scales and sums by the lanes
            int got = 1;
            if (lane == 0) got = mbar_wait(&act_empty[ab], aph ^ 1) ? 1 : 0;
            if (!__shfl_sync(0xffffffffu, got, 0)) { ok = false; break; }
            uint16_t* xs = reinterpret_cast<uint16_t*>(smem + GvSmem::act + ab * GV_ACT_BYTES);
            const int k0 = it.s0 * kTileK;
            if (lane == 0) mbar_expect_tx(&act_full[ab], it.n * it.kn * 2);
            __syncwarp();
            if (lane < it.n) {   // one row per lane, all issued at once
                const int r = lane;
                const int src = GATE_UP ? (it.sh ? it.row0 + r - a.shared_base : a.pair[it.row0 + r] / a.k) : it.row0 + r;
                bulk_load(xs + r * GV_XLD, a.act + (size_t)src * a.act_ld + k0, it.kn * 2, &act_full[ab]);
            }
            if (++ab == 2) { ab = 0; aph ^= 1; }
            // the item's weight tiles
            if (lane == 0) {
                for (int s = 0; s < it.slabs; ++s) {
                    if (!mbar_wait(&w_empty[ws], wph ^ 1)) { ok = false; break; }
                    mbar_expect_tx(&w_full[ws], kTileBytes);
                    bulk_load(smem + GvSmem::w + ws * kTileBytes, it.wband + (size_t)(it.s0 + s) * kTileBytes, kTileBytes,
                              &w_full[ws]);
                    if (++ws == GV_WSTAGES) { ws = 0; wph ^= 1; }
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            ws = __shfl_sync(0xffffffffu, ws, 0);
            wph = __shfl_sync(0xffffffffu, wph, 0);
        }
        if (!ok && lane == 0) atomicCAS(a.err, 0, FM_ETIMEOUT);
        // drain: every issued copy lands before the CTA can exit
        if (lane == 0) {
            for (int i = 0; i < GV_WSTAGES; ++i) mbar_wait(&w_full[i], i < ws ? wph : wph ^ 1);
            for (int i = 0; i < 2; ++i) mbar_wait(&act_full[i], i < ab ? aph : aph ^ 1);
        }
    } else {
        // ------------------------------------------------------------ consumer warps
        // Two groups of 8 warps take alternate slab pairs of each item (two independent chains of
        // barrier waits, shared loads and MMAs per SM); group 1 hands its sums to group 0 at the end.
        const int g = lane >> 2, c = lane & 3;
        const int grp = warp >> 3;
        const int rg = warp & 3, blk = (warp >> 2) & 1;    // rows 32 rg .. 32 rg + 31, block blk of each slab
        float2* tab = reinterpret_cast<float2*>(smem + GvSmem::tab) + warp * 64;
        float* xch2 = reinterpret_cast<float*>(smem + GvSmem::xch2);
        int ab = 0;
        uint32_t aph = 0;
        int sc0 = 0;   // running slab index of the item's first slab (the producer's fill order)
        for (int i = blockIdx.x; i < n_items; i += gridDim.x) {
            const GvItem it = gv_decode(a, i, KC);
            bool ok = __all_sync(0xffffffffu, mbar_wait(&act_full[ab], aph));
            const uint16_t* xs = reinterpret_cast<const uint16_t*>(smem + GvSmem::act + ab * GV_ACT_BYTES);
            float acc2[2][4] = {};
            for (int s = 2 * grp; s < it.slabs && ok; s += 2 * GV_GROUPS) {
                const int ws = (sc0 + s) % GV_WSTAGES;
                const uint32_t wph = ((sc0 + s) / GV_WSTAGES) & 1;
                if (s + 1 == it.slabs) {   // an odd last slab
                    if (!__all_sync(0xffffffffu, mbar_wait(&w_full[ws], wph))) { ok = false; break; }
                    const uint8_t* t1[1] = {smem + GvSmem::w + ws * kTileBytes};
                    gv_blocks<1>(t1, xs, tab, s, blk, rg, lane, acc2);
                    if (lane == 0) mbar_arrive(&w_empty[ws]);
                    break;
                }
                // two slabs at a time: independent chains
                const int ws1 = (sc0 + s + 1) % GV_WSTAGES;
                const uint32_t wph1 = ((sc0 + s + 1) / GV_WSTAGES) & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&w_full[ws], wph) && mbar_wait(&w_full[ws1], wph1))) {
                    ok = false;
                    break;
                }
                const uint8_t* tiles[2] = {smem + GvSmem::w + ws * kTileBytes, smem + GvSmem::w + ws1 * kTileBytes};
                gv_blocks<2>(tiles, xs, tab, s, blk, rg, lane, acc2);
                if (lane == 0) {
                    mbar_arrive(&w_empty[ws]);
                    mbar_arrive(&w_empty[ws1]);
                }
            }
            sc0 += it.slabs;
            __syncwarp();
            if (lane == 0) mbar_arrive(&act_empty[ab]);
            if (++ab == 2) { ab = 0; aph ^= 1; }
            if (!ok) s_abort = 1;
            named_bar(1, 32 * GV_CONSUMERS);
            if (s_abort) break;
            // C fragments: acc2[mt][0..1] = tile row 32 rg + 16 mt + g, tokens 2c, 2c+1; [2..3] = row +8.
            // As 8 values h = 2 mt + (row half), token 2c + (h & 1): rows trs[h >> 1]. Group 1 hands its
            // sums to group 0, then the block-1 warps to the block-0 warps, which own the rows from here on.
            float acc[8];
#pragma unroll
            for (int h = 0; h < 8; ++h) acc[h] = acc2[h >> 2][h & 3];
            const int trs[4] = {rg * 32 + g, rg * 32 + g + 8, rg * 32 + 16 + g, rg * 32 + 24 + g};
            if (grp == 1) {
#pragma unroll
                for (int h = 0; h < 8; ++h) xch2[(blk * 128 + trs[h >> 1]) * kGemvRows + 2 * c + (h & 1)] = acc[h];
            }
            named_bar(1, 32 * GV_CONSUMERS);
            if (grp == 0) {
#pragma unroll
                for (int h = 0; h < 8; ++h) acc[h] += xch2[(blk * 128 + trs[h >> 1]) * kGemvRows + 2 * c + (h & 1)];
            }
            if (grp == 0 && blk == 1) {
#pragma unroll
                for (int h = 0; h < 8; ++h) xch[trs[h >> 1] * kGemvRows + 2 * c + (h & 1)] = acc[h];
            }
            named_bar(1, 32 * GV_CONSUMERS);
            const bool owner = grp == 0 && blk == 0;
            if (owner) {
#pragma unroll
                for (int h = 0; h < 8; ++h) acc[h] += xch[trs[h >> 1] * kGemvRows + 2 * c + (h & 1)];
            }
            named_bar(1, 32 * GV_CONSUMERS);
            const int F = it.sh ? a.F_shared : a.F_routed;
            const int ncols = GATE_UP ? 2 * F : a.H;
            auto colof = [&](int tr) {
                return GATE_UP ? (tr < 64 ? it.bnd * 64 + tr : F + it.bnd * 64 + tr - 64) : it.bnd * kTileRows + tr;
            };
            if (KC > 1) {
                float* part = a.part + (size_t)it.kc * a.part_rows * ncols;
#pragma unroll
                for (int h = 0; h < 8; ++h) {
                    const int t = 2 * c + (h & 1);
                    if (owner && t < it.n) part[(size_t)(it.row0 + t) * ncols + colof(trs[h >> 1])] = acc[h];
                }
                __threadfence();
                named_bar(1, 32 * GV_CONSUMERS);
                if (threadIdx.x == 0) s_last = atomicAdd(&a.done[it.slot], 1) == KC - 1;
                named_bar(1, 32 * GV_CONSUMERS);
                if (!s_last) continue;
                __threadfence();
#pragma unroll
                for (int h = 0; h < 8; ++h) {
                    const int t = 2 * c + (h & 1);
                    if (owner && t < it.n) {
                        float v = 0.f;
                        for (int q = 0; q < KC; ++q)
                            v += __ldcg(a.part + (size_t)q * a.part_rows * ncols + (size_t)(it.row0 + t) * ncols + colof(trs[h >> 1]));
                        acc[h] = v;
                    }
                }
            }
            if (GATE_UP) {
                // up rows (rg 2-3) hand their sums to the gate rows (rg 0-1); h = bf16(silu(g) * u)
                if (owner && rg >= 2) {
#pragma unroll
                    for (int h = 0; h < 8; ++h) xch[(trs[h >> 1] - 64) * kGemvRows + 2 * c + (h & 1)] = acc[h];
                }
                named_bar(1, 32 * GV_CONSUMERS);
                if (owner && rg < 2) {
#pragma unroll
                    for (int h = 0; h < 8; ++h) {
                        const int t = 2 * c + (h & 1), tr = trs[h >> 1];
                        const uint16_t hb = f32_to_bf16_bits(silu_f(acc[h]) * xch[tr * kGemvRows + t]);
                        if (t < it.n) a.h_out[(size_t)(it.row0 + t) * a.h_ld + it.bnd * 64 + tr] = hb;
                    }
                }
                named_bar(1, 32 * GV_CONSUMERS);
            } else if (owner) {
#pragma unroll
                for (int h = 0; h < 8; ++h) {
                    const int t = 2 * c + (h & 1);
                    if (t < it.n) a.y_out[(size_t)(it.row0 + t) * a.H + colof(trs[h >> 1])] = acc[h];
                }
            }
        }
        if (s_abort && threadIdx.x == 0) atomicCAS(a.err, 0, FM_ETIMEOUT);
    }
    __syncthreads();
}

// ------------------------------------------------------------------ launchers
int launch_dispatch_small(const int32_t* idx, int P, int e_begin, int e_local, int shared_base, int shared_rows,
                          int* counts, int* offsets, int* pos, int* pair, int* gu_list, int gu_bands, int gu_bands_shared,
                          int gu_slabs, int* dn_list, int dn_bands, int dn_slabs, int dn_slabs_shared, int* err,
                          cudaStream_t st) {
    const size_t sm = (size_t)(e_local * 33 + 32) * 4;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(dispatch_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        attr = true;
    }
    dispatch_small_kernel<<<1, kDispSmallThreads, sm, st>>>(idx, P, e_begin, e_local, shared_base, shared_rows, counts,
                                                           offsets, pos, pair, gu_list, gu_bands, gu_bands_shared,
                                                           gu_slabs, dn_list, dn_bands, dn_slabs, dn_slabs_shared, err);
    FM_LAUNCH_CHECK("dispatch_small");
    return FM_OK;
}

static int gemv_grid(int max_items) {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return max_items < n ? max_items : n;
}

int launch_gemv(bool gate_up, const GemvLaunch& L, cudaStream_t st) {
    if (L.max_items <= 0) return FM_OK;
    GemvArgs a{};
    a.list = L.list;
    a.w_routed = L.w_routed;
    a.w_routed_stride = L.w_routed_stride;
    a.w_shared = L.w_shared;
    a.shared_group = L.shared_group;
    a.K_routed = L.K_routed;
    a.K_shared = L.K_shared;
    a.act = L.act;
    a.act_ld = L.act_ld;
    a.pair = L.pair;
    a.k = L.k;
    a.shared_base = L.shared_base;
    a.part = L.part;
    a.part_rows = L.part_rows;
    a.done = L.done;
    a.h_out = L.h_out;
    a.h_ld = L.h_ld;
    a.F_routed = L.F_routed;
    a.F_shared = L.F_shared;
    a.y_out = L.y_out;
    a.H = L.H;
    a.err = L.err;
    const int grid = gemv_grid(L.max_items);
    if (gate_up) {
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(gemv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, GvSmem::total);
            attr = true;
        }
        gemv_kernel<true><<<grid, GV_THREADS, GvSmem::total, st>>>(a);
    } else {
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(gemv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, GvSmem::total);
            attr = true;
        }
        gemv_kernel<false><<<grid, GV_THREADS, GvSmem::total, st>>>(a);
    }
    FM_LAUNCH_CHECK(gate_up ? "gemv<gate_up>" : "gemv<down>");
    return FM_OK;
}

}  // namespace fm
