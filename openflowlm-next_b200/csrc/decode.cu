// Decode-size path (T <= 128 tokens, T * top_k <= 1024): single-CTA dispatch that also builds the GEMV
// work lists, and the bandwidth-bound grouped Q4_1 GEMV.
//
// GEMV: a work item is (group, 128-row band, up to 8 sorted rows, K chunk). Each SM runs four
// independent CTAs of one producer warp + four consumer warps. The producer streams the item's slabs
// into a ring of 8 stages, each one 5120-byte weight tile (one bulk copy) plus the item's activation
// rows for the same 64 K (one 128-byte bulk copy per row). Consumer warp j owns tile rows 16j..16j+15
// and 64+16j..64+16j+15 over the whole K chunk: for gate/up these are the gate and up rows of the same
// 16 features, so SwiGLU happens in registers and no warp waits for another.
// The tensor core multiplies the raw codes, never dequantised weights: the A operand is 128 + q as bf16
// (exact; one byte permute per two codes, one 32-bit load per fragment thanks to the tile's fragment
// byte order), the B operand the bf16 activations, so per 32-value block C = sum (128 + q) x exactly in
// f32, and the block's exact fp16 scale d and min m are applied after the MMA:
//   y += d * C + (m - 128 d) * X,   X = sum of the block's activations (an all-ones MMA),
// i.e. the oracle's exact dequantisation (q4_1_pack.py:104-109) with only f32 roundings. With few tokens
// per item the MMA's 8 columns hold several blocks (column = token x block phase), so the per-block
// scale work is done once per 8 / tokens blocks instead of per block.
// K is split into chunks only when there are fewer than two items per SM. gate/up: the last warp to
// finish a (slot, rows) reduces the chunks' partial sums in chunk order (deterministic), then applies
// SwiGLU; down: chunks add into the y rows with red.add (the gate/up kernel clears them first).
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

// Block-wide (1024 threads) exclusive scan of two ints per thread (x and y scanned independently) and
// their block totals; sh holds 64 ints.
__device__ int2 block_exclusive_scan2_1024(int2 v, int* sh, int2* tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int2 x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ya = __shfl_up_sync(0xffffffffu, x.x, o), yb = __shfl_up_sync(0xffffffffu, x.y, o);
        if (lane >= o) { x.x += ya; x.y += yb; }
    }
    __syncthreads();
    if (lane == 31) { sh[warp] = x.x; sh[32 + warp] = x.y; }
    __syncthreads();
    if (warp == 0) {
        int sa = sh[lane], sb = sh[32 + lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int ya = __shfl_up_sync(0xffffffffu, sa, o), yb = __shfl_up_sync(0xffffffffu, sb, o);
            if (lane >= o) { sa += ya; sb += yb; }
        }
        sh[lane] = sa;
        sh[32 + lane] = sb;
    }
    __syncthreads();
    const int2 r = make_int2((warp ? sh[warp - 1] : 0) + x.x - v.x, (warp ? sh[31 + warp] : 0) + x.y - v.y);
    *tot = make_int2(sh[31], sh[63]);
    __syncthreads();
    return r;
}

// K chunks per item: the smallest divisor of the slab counts (at least two slabs per chunk, at most
// kc_cap chunks) that gives `target` items (two per SM), else the largest such divisor. Splits
// are kept few: each costs a round trip of n x 128 partial sums through L2, a completion counter and
// the ramp of another item, measured dearer than the load imbalance they remove.
__device__ int choose_chunks(int base_items, int slabs, int slabs_other, int kc_cap, int target) {
    int best = 1;
    if (base_items >= target) return 1;
    for (int kc = 2; kc <= kc_cap; ++kc) {
        if (slabs % kc || slabs / kc < 2) continue;
        if (slabs_other && (slabs_other % kc || slabs_other / kc < 2)) continue;
        best = kc;
        if (base_items * kc >= target) break;
    }
    return best;
}

__global__ void __launch_bounds__(kDispSmallThreads) dispatch_small_kernel(
    const int32_t* __restrict__ idx, int P, int e_begin, int e_local, int shared_base, int shared_rows,
    int* __restrict__ counts, int* __restrict__ offsets, int* __restrict__ pos, int* __restrict__ pair,
    int* __restrict__ gu_list, int gu_bands, int gu_bands_shared, int gu_slabs, int* __restrict__ dn_list, int dn_bands,
    int dn_slabs, int dn_slabs_shared, int kc_cap, int split, int target, int clear, int* __restrict__ done, int* __restrict__ err) {
    extern __shared__ int sm[];
    int* cnt = sm;                                  // [e_local]
    int* wcnt = cnt + e_local;                      // [32][e_local]
    int* scan_sh = wcnt + 32 * e_local;             // [64]
    int* off_s = scan_sh + 64;                      // [e_local + 1] group row offsets
    int* gu0 = off_s + e_local + 1;                 // [e_local + 2] first GEMV slot of each group (gate/up)
    int* dn0 = gu0 + e_local + 2;                   // [e_local + 2] (down)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_launch_dependents();
    // this call's status words (bad ids, GEMV timeouts), unless the caller cleared them before its router
    if (clear && threadIdx.x < 4) err[threadIdx.x] = 0;
    __syncthreads();
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
            off_s[threadIdx.x] = ex;
        }
        if (threadIdx.x == 0) {
            counts[e_local] = shared_rows;
            offsets[e_local] = scan_sh[31];
            offsets[e_local + 1] = shared_base;
            off_s[e_local] = shared_base;
        }
        __syncthreads();
    }
    if (e >= 0) {
        const int b = off_s[e] + wcnt[warp * e_local + e] + rank;
        pos[p] = b;
        pair[b] = p;
    } else if (p < P) {
        pos[p] = -1;
    }
    // GEMV work lists. Group g (G <= 1024: the local experts, then the shared expert) has ceil(rows / 8)
    // row chunks x its bands of slots, each slot kc K-chunk items; slots are numbered group-major. All
    // threads write the items: item e -> slot e / kc, found by a binary search over the groups' first slots.
    const int G = e_local + (shared_rows > 0 ? 1 : 0);
    const int gi = threadIdx.x;
    int c_g = 0, bands_g = 0, tt = 0;
    if (gi < G) {
        c_g = gi < e_local ? cnt[gi] : shared_rows;
        bands_g = gi < e_local ? gu_bands : gu_bands_shared;
        tt = (c_g + kGemvRows - 1) / kGemvRows;
    }
    const int bgu = tt * bands_g, bdn = tt * dn_bands;
    int2 tot;
    const int2 slot = block_exclusive_scan2_1024(make_int2(bgu, bdn), scan_sh, &tot);
    const int tot_gu = tot.x, tot_dn = tot.y, slot_gu = slot.x, slot_dn = slot.y;
    // K chunks: their count follows the call's item count (so a token's sums would depend on the other
    // tokens of the call) and the down GEMM adds its chunks into y with red.add (an unfixed order): both
    // off in the fixed-order mode
    const int kc_gu = split ? choose_chunks(tot_gu, gu_slabs, 0, kc_cap, target) : 1;
    const int kc_dn = split ? choose_chunks(tot_dn, dn_slabs, shared_rows > 0 ? dn_slabs_shared : 0, kc_cap, target) : 1;
    if (gi <= G) {
        gu0[gi] = gi < G ? slot_gu : tot_gu;
        dn0[gi] = gi < G ? slot_dn : tot_dn;
    }
    // the GEMV's per-(item slot, warp) completion counters start at zero
    for (int i = threadIdx.x; i < tot_gu * kGemvWarps; i += blockDim.x) done[i] = 0;
    __syncthreads();
    auto emit = [&](int* list, const int* first, int total, int kc, int bands_routed, int bands_shared) {
        for (int e = threadIdx.x; e < total * kc; e += blockDim.x) {
            const int slot = e / kc, q = e - slot * kc;
            int lo = 0, hi = G - 1;   // last group whose first slot <= slot
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (first[mid] <= slot) lo = mid; else hi = mid - 1;
            }
            const int grp = lo, local = slot - first[grp];
            const int bands = grp < e_local ? bands_routed : bands_shared;
            const int r = local / bands, b = local - r * bands;
            const int rows = grp < e_local ? cnt[grp] : shared_rows;
            const int n = min(kGemvRows, rows - r * kGemvRows);
            reinterpret_cast<int4*>(list + 4)[e] = make_int4(grp | (b << 16), off_s[grp] + r * kGemvRows, n | (q << 16), slot);
        }
    };
    emit(gu_list, gu0, tot_gu, kc_gu, gu_bands, gu_bands_shared);
    emit(dn_list, dn0, tot_dn, kc_dn, dn_bands, dn_bands);
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
    float* part;              // [KC][part_rows][part_ld] f32 partial sums (K split)
    int part_rows, part_ld;
    int* done;                // completion counters per (item slot, consumer warp), zeroed by the dispatch
    uint16_t* h_out;          // GATE_UP final: bf16 h [rows, h_ld]
    int h_ld;
    int F_routed, F_shared;   // GATE_UP: features per matrix
    float* y_out;             // DOWN final: f32 [rows, H]; with K chunks the chunks add into it (red.add)
    int H;
    const int* dn_list;       // GATE_UP: the down list, whose K-chunk count says whether y starts at zero
    int y_rows;               // rows of y_out
    int* err;                 // FM_ETIMEOUT when a bounded wait gives up
    int tc_min;               // least token columns per item (8: one scale group per block at every n)
};

// CTA = one producer warp + GV_WARPS consumer warps working on one item at a time; GV_CTAS_PER_SM such
// CTAs share an SM, each with its own ring of GV_STAGES slabs (a 5120-byte weight tile plus the item's
// activation rows for the same 64 K).
constexpr int GV_WARPS = kGemvWarps;
constexpr int GV_THREADS = 32 * (GV_WARPS + 1);
constexpr int GV_CTAS_PER_SM = 4;
constexpr int GV_STAGES = 8;
constexpr int GV_XROW = 144;                                  // staged activation row: 64 bf16 + 16 B (bank spread)
constexpr int GV_STAGE = kTileBytes + kGemvRows * GV_XROW;    // 6272 B
struct GvSmem {
    static constexpr int zero = GV_STAGES * GV_STAGE;         // 64 zero bytes (B operand of off-phase columns)
    static constexpr int bars = zero + 64;
    static constexpr int total = bars + 2 * GV_STAGES * 8 + 128;   // + alignment slack
};

__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Shared-memory loads by 32-bit shared address (no generic-to-shared conversion per access). Volatile
// so they stay after the mbarrier waits that make the data visible.
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// (d, m - 128 d) of row `row`, block `blk` of the tile at shared address w, in f32 (d and m are exact
// fp16 values).
__device__ __forceinline__ float2 gv_scale(uint32_t w, int row, int blk) {
    const uint32_t sc = lds32(w + kTileNibBytes + row * 8 + blk * 4);
    const float d = __half2float(__ushort_as_half((unsigned short)(sc & 0xFFFF)));
    const float m = __half2float(__ushort_as_half((unsigned short)(sc >> 16)));
    return make_float2(d, fmaf(-128.f, d, m));
}

// One 16-value K step (hi = 0: values 0-15 of the block, 1: values 16-31) of the warp's two m16 row
// tiles: cb[mt] += (128 + q) x on the tensor core, cx += 1 x (the block sums of each column).
// u[mt][h]: the lane's fragment word of tile row (16 j + g + 8 h + 64 mt): low nibbles are values
// 2c, 2c+1, 2c+8, 2c+9 of the block, high nibbles the same + 16.
__device__ __forceinline__ void gv_kstep(const uint32_t (&u)[2][2], int hi, uint32_t b0, uint32_t b1, float (&cb)[2][4],
                                         float (&cx)[4]) {
    const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
        const uint32_t ta = (hi ? u[mt][0] >> 4 : u[mt][0]) & 0x0F0F0F0Fu;
        const uint32_t tb = (hi ? u[mt][1] >> 4 : u[mt][1]) & 0x0F0F0F0Fu;
        uint32_t af[4];
        af[0] = __byte_perm(ta, 0x43434343u, 0x5140);   // bf16 128 + q of values 2c, 2c+1 (row g)
        af[1] = __byte_perm(tb, 0x43434343u, 0x5140);   // row g + 8
        af[2] = __byte_perm(ta, 0x43434343u, 0x5342);   // values 2c+8, 2c+9
        af[3] = __byte_perm(tb, 0x43434343u, 0x5342);
        mma_bf16(cb[mt], af, b0, b1);
    }
    mma_bf16(cx, ones, b0, b1);
}

// One item's K range for a consumer warp, TC = token columns (n <= TC <= 8). The 8 columns of the MMA
// are (token t, block phase p) with t = col % TC, p = col / TC: a lane loads its B column's activations
// only for blocks whose index within the group is p (else zeros), so one C fragment collects P = 8 / TC
// consecutive blocks without mixing them, and the exact per-block scales are applied once per group of
// P blocks: acc += d C + (m - 128 d) X. A group's stages are released after its scales are read.
template <int TC>
__device__ __forceinline__ bool gv_item(uint8_t* smem, uint64_t* full, uint64_t* empty, int& st, uint32_t& ph, int slabs,
                                        int j, int lane, float (&acc)[2][4]) {
    constexpr int P = 8 / TC;
    constexpr int GS = P >= 2 ? P / 2 : 1;    // slabs per scale group
    const int g = lane >> 2, c = lane & 3;
    const int bt = g % TC, bp = g / TC;       // this lane's B column: token bt, block phase bp
    const int r0 = 16 * j + g;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t zero = sbase + GvSmem::zero + 4 * c;
    for (int s0 = 0; s0 < slabs; s0 += GS) {
        const int gs = min(GS, slabs - s0);
        const int st0 = st;
        float cb[2][4] = {}, cx[4] = {};
#pragma unroll
        for (int q = 0; q < GS; ++q) {
            if (q < gs) {
                if (!__all_sync(0xffffffffu, mbar_wait(&full[st], ph))) return false;
                const uint32_t w = sbase + st * GV_STAGE;
                const uint32_t wr = w + r0 * 32 + 4 * c;                       // row r0's fragment word
                const uint32_t xr = w + kTileBytes + bt * GV_XROW + 4 * c;     // this lane's B column
#pragma unroll
                for (int blk = 0; blk < 2; ++blk) {
                    const bool on = P == 1 || bp == (2 * q + blk) % P;
                    const uint32_t xb = on ? xr + blk * 64 : zero;
                    uint32_t u[2][2];
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                        for (int h = 0; h < 2; ++h) u[mt][h] = lds32(wr + (64 * mt + 8 * h) * 32 + blk * 16);
#pragma unroll
                    for (int hi = 0; hi < 2; ++hi) {
                        const uint32_t b0 = lds32(xb + hi * 32);
                        const uint32_t b1 = lds32(xb + hi * 32 + 16);
                        gv_kstep(u, hi, b0, b1, cb, cx);
                    }
                    if (P == 1) {   // every column is this block: apply its scales now
#pragma unroll
                        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const float2 sc = gv_scale(w, r0 + 64 * mt + 8 * h, blk);
#pragma unroll
                                for (int cc = 0; cc < 2; ++cc) {
                                    acc[mt][2 * h + cc] = fmaf(sc.x, cb[mt][2 * h + cc], fmaf(sc.y, cx[cc], acc[mt][2 * h + cc]));
                                    cb[mt][2 * h + cc] = 0.f;
                                }
                            }
                        cx[0] = cx[1] = cx[2] = cx[3] = 0.f;
                    }
                }
                if (P == 1) {   // release the stage (its next fill is an async-proxy copy)
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[st]);
                }
                if (++st == GV_STAGES) { st = 0; ph ^= 1; }
            }
        }
        if (P > 1) {
            // this lane's C columns 2c and 2c+1 hold block phases p0 and p1 of the group (the same
            // phase unless TC == 1); a short last group lacks the phases past its slabs
#pragma unroll
            for (int cc = 0; cc < (TC == 1 ? 2 : 1); ++cc) {
                const int pc = (2 * c + cc) / TC;
                if (pc / 2 < gs) {
                    int sidx = st0 + pc / 2;
                    if (sidx >= GV_STAGES) sidx -= GV_STAGES;
                    const uint32_t w = sbase + sidx * GV_STAGE;
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float2 sc = gv_scale(w, r0 + 64 * mt + 8 * h, pc & 1);
#pragma unroll
                            for (int e = cc; e < 2; e += (TC == 1 ? 2 : 1))
                                acc[mt][2 * h + e] = fmaf(sc.x, cb[mt][2 * h + e], fmaf(sc.y, cx[e], acc[mt][2 * h + e]));
                        }
                }
            }
            // release the group's stages: every load from them has delivered its value (the
            // accumulators depend on them), and the fence orders these reads before the producer's
            // next bulk copies (async proxy) into the same stages
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0)
                for (int q = 0; q < gs; ++q) mbar_arrive(&empty[(st0 + q) % GV_STAGES]);
        }
    }
    return true;
}

struct GvItem {
    int grp, bnd, row0, n, kc, slot, slabs, s0;
    bool sh;
    const uint8_t* wband;
};

__device__ __forceinline__ int4 gv_entry(const GemvArgs& a, int i, int n_items) {
    return i < n_items ? __ldg(reinterpret_cast<const int4*>(a.list + 4) + i) : make_int4(0, 0, 0, 0);
}

// Sorted row -> row of the activation matrix (GATE_UP: the token; DOWN: the sorted h row).
template <bool GATE_UP>
__device__ __forceinline__ int gv_src_row(const GemvArgs& a, int4 e, int lane) {
    const int n = e.z & 0xFFFF, row = e.y + lane;
    if (lane >= n) return 0;
    if (!GATE_UP) return row;
    return (e.x & 0xFFFF) == a.shared_group ? row - a.shared_base : __ldg(a.pair + row) / a.k;
}

__device__ __forceinline__ GvItem gv_decode(const GemvArgs& a, int4 it, int KC) {
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
    r.wband = (r.sh ? a.w_shared : a.w_routed + (size_t)r.grp * a.w_routed_stride) + (size_t)r.bnd * (K / kTileK) * kTileBytes;
    return r;
}

// Items: (group, 128-row band, up to 8 sorted rows, K chunk). Consumer warp j owns tile rows
// 16j..16j+15 (m16 tile 0) and 64+16j..64+16j+15 (m16 tile 1): for GATE_UP the gate and up rows of the
// same 16 features, so SwiGLU needs no exchange between warps; every warp covers the item's whole K
// chunk, so no reduction between warps either. The last warp to finish a (slot, warp) over the K chunks
// reduces them in chunk order (deterministic).
template <bool GATE_UP>
__global__ void __launch_bounds__(GV_THREADS, GV_CTAS_PER_SM) gemv_kernel(GemvArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + GvSmem::bars);
    uint64_t* empty = full + GV_STAGES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < GV_STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], GV_WARPS);
        }
        mbar_fence_init();
    }
    if (threadIdx.x < 16) reinterpret_cast<uint32_t*>(smem + GvSmem::zero)[threadIdx.x] = 0u;
    __syncthreads();
    pdl_wait();
    pdl_launch_dependents();
    // the item count and this CTA's first entry load together (the entry's slot exists: the grid is no
    // larger than the list's capacity); the entry is dropped when it lies past the count
    const int4 first = __ldg(reinterpret_cast<const int4*>(a.list + 4) + blockIdx.x);
    const int n_items = a.list[0], KC = a.list[1];
    const int4 e_first = (int)blockIdx.x < n_items ? first : make_int4(0, 0, 0, 0);
    if (GATE_UP && a.dn_list[1] > 1) {   // the down GEMM will add its K chunks into y: clear it first
        float4* y4 = reinterpret_cast<float4*>(a.y_out);
        const long long n4 = (long long)a.y_rows * a.H / 4;
        for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x)
            y4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    if (warp == GV_WARPS) {
        // ------------------------------------------------------------ producer warp
        int st = 0;
        uint32_t ph = 0;
        bool ok = true;
        // list entries two items ahead and source rows one item ahead are in flight while an item's
        // slabs are issued
        const int G = gridDim.x;
        int4 e0 = e_first, e1 = gv_entry(a, blockIdx.x + G, n_items);
        int row0 = gv_src_row<GATE_UP>(a, e0, lane);
        for (int i = blockIdx.x; i < n_items && ok; i += G) {
            const int4 e2 = gv_entry(a, i + 2 * G, n_items);
            const int row1 = gv_src_row<GATE_UP>(a, e1, lane);
            const GvItem it = gv_decode(a, e0, KC);
            // lane r < n: token row r of the item, from the chunk's first K
            const uint16_t* src = a.act + (size_t)row0 * a.act_ld + (size_t)it.s0 * kTileK;
            e0 = e1;
            e1 = e2;
            row0 = row1;
            for (int s = 0; s < it.slabs; ++s) {
                int got = 1;
                if (lane == 0) got = mbar_wait(&empty[st], ph ^ 1) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, got, 0)) {
                    ok = false;
                    break;
                }
                uint8_t* stage = smem + st * GV_STAGE;
                if (lane == 0) {
                    mbar_expect_tx(&full[st], kTileBytes + it.n * kTileK * 2);
                    bulk_load(stage, it.wband + (size_t)(it.s0 + s) * kTileBytes, kTileBytes, &full[st]);
                }
                __syncwarp();
                if (lane < it.n) bulk_load(stage + kTileBytes + lane * GV_XROW, src + s * kTileK, kTileK * 2, &full[st]);
                if (++st == GV_STAGES) { st = 0; ph ^= 1; }
            }
        }
        if (!ok && lane == 0) atomicCAS(a.err, 0, FM_ETIMEOUT);
        // drain: every issued copy lands before the CTA can exit
        if (lane == 0)
            for (int i = 0; i < GV_STAGES; ++i) mbar_wait(&full[i], i < st ? ph : ph ^ 1);
    } else {
        // ------------------------------------------------------------ consumer warps
        const int j = warp, g = lane >> 2, c = lane & 3;
        int st = 0;
        uint32_t ph = 0;
        bool ok = true;
        int4 e0 = e_first;
        for (int i = blockIdx.x; i < n_items; i += gridDim.x) {
            const int4 e1 = gv_entry(a, i + gridDim.x, n_items);   // the next item's entry, in flight
            const GvItem it = gv_decode(a, e0, KC);
            e0 = e1;
            float acc[2][4] = {};
            // token columns: fewer tokens leave room for several blocks per MMA column group (gv_item),
            // which changes the order of a token's sums with the item's token count; tc_min = 8 keeps
            // one order for every count (the fixed-order mode)
            const int tc = max(a.tc_min, it.n <= 1 ? 1 : it.n <= 2 ? 2 : it.n <= 4 ? 4 : 8);
            switch (tc) {
                case 1: ok = gv_item<1>(smem, full, empty, st, ph, it.slabs, j, lane, acc); break;
                case 2: ok = gv_item<2>(smem, full, empty, st, ph, it.slabs, j, lane, acc); break;
                case 4: ok = gv_item<4>(smem, full, empty, st, ph, it.slabs, j, lane, acc); break;
                default: ok = gv_item<8>(smem, full, empty, st, ph, it.slabs, j, lane, acc); break;
            }
            if (!ok) break;
            // per (row, token) sums: add the lane's columns of the same token (other block phases)
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                if (tc == 1) {
                    acc[mt][0] += acc[mt][1];
                    acc[mt][2] += acc[mt][3];
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if (tc <= 2) acc[mt][e] += __shfl_xor_sync(0xffffffffu, acc[mt][e], 1);
                    if (tc <= 4) acc[mt][e] += __shfl_xor_sync(0xffffffffu, acc[mt][e], 2);
                }
            }
            // lane c owns tokens 2c, 2c+1 (tc >= 2) or token 0 (tc == 1, lane c = 0, column 0)
            bool own[2];
#pragma unroll
            for (int cc = 0; cc < 2; ++cc)
                own[cc] = (tc == 1 ? (c == 0 && cc == 0) : (2 * c < tc)) && 2 * c + cc < it.n;
            const int F = it.sh ? a.F_shared : a.F_routed;
            const int ncols = a.part_ld;   // one row stride for every group (F and F_s may differ)
            auto colof = [&](int mt, int h) {
                const int r = 16 * j + g + 8 * h;
                return GATE_UP ? mt * F + it.bnd * 64 + r : it.bnd * kTileRows + 64 * mt + r;
            };
            if (!GATE_UP && KC > 1) {   // y rows were cleared by the gate/up kernel: add this chunk
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc)
                        if (own[cc]) {
                            const size_t row = (size_t)(it.row0 + 2 * c + cc);
                            atomicAdd(a.y_out + row * a.H + colof(0, h), acc[0][2 * h + cc]);
                            atomicAdd(a.y_out + row * a.H + colof(1, h), acc[1][2 * h + cc]);
                        }
                continue;
            }
            if (KC > 1) {
                float* part = a.part + (size_t)it.kc * a.part_rows * ncols;
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc)
                            if (own[cc]) part[(size_t)(it.row0 + 2 * c + cc) * ncols + colof(mt, h)] = acc[mt][2 * h + cc];
                __threadfence();
                __syncwarp();
                int last = 0;
                if (lane == 0) last = atomicAdd(&a.done[it.slot * GV_WARPS + j], 1) == KC - 1;
                if (!__shfl_sync(0xffffffffu, last, 0)) continue;
                __threadfence();
                // each owned value's KC partial sums, added in chunk order; the loads of four chunks for
                // all of the lane's values are issued before their adds, so the reduction costs
                // ceil(KC / 4) L2 round trips rather than one per partial sum
                const size_t zs = (size_t)a.part_rows * ncols;
                float v[2][2][2] = {};
                for (int q0 = 0; q0 < KC; q0 += 4) {
                    float pv[4][2][2][2];
#pragma unroll
                    for (int u = 0; u < 4; ++u)
#pragma unroll
                        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                            for (int h = 0; h < 2; ++h)
#pragma unroll
                                for (int cc = 0; cc < 2; ++cc)
                                    pv[u][mt][h][cc] = own[cc] && q0 + u < KC
                                                           ? __ldcg(a.part + (size_t)(q0 + u) * zs +
                                                                    (size_t)(it.row0 + 2 * c + cc) * ncols + colof(mt, h))
                                                           : 0.f;
#pragma unroll
                    for (int u = 0; u < 4; ++u)
#pragma unroll
                        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                            for (int h = 0; h < 2; ++h)
#pragma unroll
                                for (int cc = 0; cc < 2; ++cc)
                                    if (q0 + u < KC) v[mt][h][cc] += pv[u][mt][h][cc];
                }
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc)
                            if (own[cc]) acc[mt][2 * h + cc] = v[mt][h][cc];
            }
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    if (!own[cc]) continue;
                    const size_t row = (size_t)(it.row0 + 2 * c + cc);
                    if (GATE_UP) {
                        const float hv = silu_f(acc[0][2 * h + cc]) * acc[1][2 * h + cc];   // h = bf16(silu(g) u)
                        a.h_out[row * a.h_ld + it.bnd * 64 + 16 * j + g + 8 * h] = f32_to_bf16_bits(hv);
                    } else {
                        a.y_out[row * a.H + colof(0, h)] = acc[0][2 * h + cc];
                        a.y_out[row * a.H + colof(1, h)] = acc[1][2 * h + cc];
                    }
                }
        }
        if (!ok && lane == 0) atomicCAS(a.err, 0, FM_ETIMEOUT);
    }
}

// ------------------------------------------------------------------ launchers
// Past 32 tokens there are items enough for every CTA slot, and no K split (no partial-sum buffer).
int gemv_chunk_cap(int T) {
    if (T > 32) return 1;
    const int cap = T <= 4 ? 16 : 64 / T;
    return cap < 2 ? 2 : cap;
}

int launch_dispatch_small(const int32_t* idx, int P, int e_begin, int e_local, int shared_base, int shared_rows,
                          int* counts, int* offsets, int* pos, int* pair, int* gu_list, int gu_bands, int gu_bands_shared,
                          int gu_slabs, int* dn_list, int dn_bands, int dn_slabs, int dn_slabs_shared, int kc_cap, int split,
                          int clear, int* done, int* err, cudaStream_t st) {
    const size_t sm = (size_t)(e_local * 33 + 64 + 3 * (e_local + 2)) * 4;
    // the limit for the largest group count (e_local < 1024) at once, so no later call (one being
    // captured into a graph, say) has to raise it again
    if (cudaError_t e = raise_smem_limit((const void*)dispatch_small_kernel, 160 * 1024))
        return cuda_status(e, "dispatch_small smem");
    // K chunks are added until a call has two items per SM (half the CTA slots): filling every slot
    // measured slower at 1-8 tokens, its extra chunks costing more in partial sums and second rounds of
    // items than they add in parallel loads
    const int target = 2 * device_sm_count();
    FM_LAUNCH_PDL("dispatch_small", dispatch_small_kernel, dim3(1), dim3(kDispSmallThreads), sm, st, idx, P, e_begin, e_local,
                  shared_base, shared_rows, counts, offsets, pos, pair, gu_list, gu_bands, gu_bands_shared, gu_slabs, dn_list,
                  dn_bands, dn_slabs, dn_slabs_shared, kc_cap, split, target, clear, done, err);
    return FM_OK;
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
    a.part_ld = L.part_ld;
    a.done = L.done;
    a.h_out = L.h_out;
    a.h_ld = L.h_ld;
    a.F_routed = L.F_routed;
    a.F_shared = L.F_shared;
    a.y_out = L.y_out;
    a.H = L.H;
    a.dn_list = L.dn_list;
    a.y_rows = L.y_rows;
    a.err = L.err;
    a.tc_min = L.tc_min;
    const int slots = GV_CTAS_PER_SM * device_sm_count();
    const int grid = L.max_items < slots ? L.max_items : slots;
    const void* fn = gate_up ? (const void*)gemv_kernel<true> : (const void*)gemv_kernel<false>;
    if (cudaError_t e = raise_smem_limit(fn, GvSmem::total)) return cuda_status(e, "gemv smem");
    if (gate_up)
        FM_LAUNCH_PDL("gemv<gate_up>", gemv_kernel<true>, dim3(grid), dim3(GV_THREADS), GvSmem::total, st, a);
    else
        FM_LAUNCH_PDL("gemv<down>", gemv_kernel<false>, dim3(grid), dim3(GV_THREADS), GvSmem::total, st, a);
    return FM_OK;
}

}  // namespace fm
