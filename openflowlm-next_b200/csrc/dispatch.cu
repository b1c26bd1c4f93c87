// Token dispatch: per-expert counts (histogram), exclusive scan, stable permutation, gather.
//
// The reference builds per-expert "owed" lists on the host in token-then-slot order and visits
// experts in ascending order (src/open_qwen36/core.cpp:5155-5165), then gathers the visited tokens'
// rows as bf16 (core.cpp:5180-5207). Here the same order is a stable counting sort on the device:
//   dispatch_hist    per-chunk expert histograms (shared-memory atomics),
//   dispatch_scan    one block: per-expert counts, exclusive offsets, per-chunk bases, the GEMM work
//                    lists,
//   dispatch_scatter per chunk, stable ranks (warp match + per-warp prefix in shared memory),
//   gather_rows      x rows -> the expert-sorted bf16 activation matrix.
// Counts, offsets and permutation are integer results and match the oracle bit for bit.
#include "common.cuh"

namespace fm {

constexpr int kChunk = 2048;   // pairs per dispatch block
constexpr int kDispThreads = 256;

__global__ void __launch_bounds__(kDispThreads) dispatch_hist_kernel(const int32_t* __restrict__ idx, int P, int e_begin,
                                                                     int e_local, int E, int* __restrict__ blk_hist,
                                                                     int* __restrict__ err) {
    extern __shared__ int hist[];
    for (int e = threadIdx.x; e < e_local; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const int p0 = blockIdx.x * kChunk;
    int bad = 0;
    for (int i = threadIdx.x; i < kChunk && p0 + i < P; i += blockDim.x) {
        const int e = idx[p0 + i] - e_begin;
        if (e >= 0 && e < e_local) atomicAdd(&hist[e], 1);
        else ++bad;
    }
    if (bad) atomicAdd(err, bad);
    __syncthreads();
    for (int e = threadIdx.x; e < e_local; e += blockDim.x) blk_hist[(size_t)blockIdx.x * e_local + e] = hist[e];
}

// Work list entry: (group, band, row0, nrows). list[0] = number of entries. Row tiles outer, bands
// inner, so consecutive items share their activation rows in L2. A group's cnt rows make ceil(cnt / bn)
// tiles of equal size (rounded up to 16 rows, the MMA's N step; the last takes the rest), so that no
// tile is a sliver whose MMAs cost their issue time rather than their width.
__device__ void emit_tiles(int* list, int first, int g, int bands, int row0, int cnt, int bn) {
    const int nt = (cnt + bn - 1) / bn;
    const int step = nt > 0 ? min(bn, ((cnt + nt - 1) / nt + 15) & ~15) : bn;
    int i = first;
    for (int r = 0; r < cnt; r += step)
        for (int b = 0; b < bands; ++b, ++i) {
            int4 t = make_int4(g, b, row0 + r, min(step, cnt - r));
            reinterpret_cast<int4*>(list + 4)[i] = t;
        }
}

// One block of 1024 threads. Groups 0..e_local-1 are the routed experts, group e_local the shared
// expert (rows = shared_rows, stored after the routed capacity P).
__global__ void __launch_bounds__(1024) dispatch_scan_kernel(int* __restrict__ blk_hist, int nblk, int e_local,
                                                             int shared_base, int shared_rows, int* __restrict__ counts,
                                                             int* __restrict__ offsets, int* __restrict__ gu_list,
                                                             int gu_bands, int gu_bands_shared, int* __restrict__ dn_list,
                                                             int dn_bands, int bn) {
    __shared__ int sh[32];
    const int G = e_local + 1;
    int carry = 0, total = 0;
    // counts and per-chunk relative bases, per expert (serial over chunks)
    for (int e0 = 0; e0 < e_local; e0 += 1024) {
        const int e = e0 + threadIdx.x;
        int run = 0;
        // chunk histograms -> exclusive per-chunk prefixes, 16 chunks' loads in flight at a time
        if (e < e_local)
            for (int b0 = 0; b0 < nblk; b0 += 16) {
                int v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = b0 + j < nblk ? blk_hist[(size_t)(b0 + j) * e_local + e] : 0;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (b0 + j < nblk) {
                        blk_hist[(size_t)(b0 + j) * e_local + e] = run;
                        run += v[j];
                    }
            }
        const int ex = block_exclusive_scan(e < e_local ? run : 0, sh, &total);
        if (e < e_local) {
            counts[e] = run;
            offsets[e] = carry + ex;
            for (int b0 = 0; b0 < nblk; b0 += 16) {
                int v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = b0 + j < nblk ? blk_hist[(size_t)(b0 + j) * e_local + e] : 0;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (b0 + j < nblk) blk_hist[(size_t)(b0 + j) * e_local + e] = v[j] + carry + ex;
            }
        }
        carry += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        counts[e_local] = shared_rows;
        offsets[e_local] = carry;                 // end of the routed rows
        offsets[e_local + 1] = shared_base;       // the shared expert's rows start here
    }
    __syncthreads();
    // work lists: ceil(count / bn) row tiles per band
    int gu_carry = 0, dn_carry = 0;
    for (int g0 = 0; g0 < G; g0 += 1024) {
        const int g = g0 + threadIdx.x;
        int cnt = 0, row0 = 0;
        if (g < G) {
            cnt = counts[g];
            row0 = g == e_local ? shared_base : offsets[g];
        }
        const int rt = (cnt + bn - 1) / bn;
        const int ngu = g < G ? rt * (g == e_local ? gu_bands_shared : gu_bands) : 0;
        const int ndn = g < G ? rt * dn_bands : 0;
        int tgu = 0, tdn = 0;
        const int egu = block_exclusive_scan(ngu, sh, &tgu);
        const int edn = block_exclusive_scan(ndn, sh, &tdn);
        if (g < G && cnt > 0) {
            emit_tiles(gu_list, gu_carry + egu, g, g == e_local ? gu_bands_shared : gu_bands, row0, cnt, bn);
            emit_tiles(dn_list, dn_carry + edn, g, dn_bands, row0, cnt, bn);
        }
        gu_carry += tgu;
        dn_carry += tdn;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        gu_list[0] = gu_carry;
        dn_list[0] = dn_carry;
    }
}

// Stable ranks: the chunk is walked in rounds of 256 pairs (one per thread, in pair order).
// Within a warp, __match_any_sync gives each lane its rank among same-expert lanes; across the
// round's 8 warps, a per-warp count table in shared memory gives the prefix; `base[e]` carries the
// running position across rounds. pos[p] = sorted row (or -1), pair[row] = p.
__global__ void __launch_bounds__(kDispThreads) dispatch_scatter_kernel(const int32_t* __restrict__ idx, int P,
                                                                        int e_begin, int e_local,
                                                                        const int* __restrict__ blk_base,
                                                                        int* __restrict__ pos, int* __restrict__ pair) {
    extern __shared__ int smem[];
    int* base = smem;                       // [e_local]
    int* wcnt = smem + e_local;             // [8][e_local]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < e_local; e += blockDim.x) {
        base[e] = blk_base[(size_t)blockIdx.x * e_local + e];
        for (int w = 0; w < kDispThreads / 32; ++w) wcnt[w * e_local + e] = 0;
    }
    __syncthreads();
    const int p0 = blockIdx.x * kChunk;
    for (int r = 0; r < kChunk; r += kDispThreads) {
        const int p = p0 + r + threadIdx.x;
        int e = -1;
        if (p < P) {
            e = idx[p] - e_begin;
            if (e < 0 || e >= e_local) e = -1;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (e >= 0 && rank == 0) wcnt[warp * e_local + e] = __popc(peers);
        __syncthreads();
        if (e >= 0) {
            int b = base[e] + rank;
            for (int w = 0; w < warp; ++w) b += wcnt[w * e_local + e];
            pos[p] = b;
            pair[b] = p;
        } else if (p < P) {
            pos[p] = -1;
        }
        __syncthreads();
        for (int x = threadIdx.x; x < e_local; x += blockDim.x) {
            int s = 0;
            for (int w = 0; w < kDispThreads / 32; ++w) {
                s += wcnt[w * e_local + x];
                wcnt[w * e_local + x] = 0;
            }
            base[x] += s;
        }
        __syncthreads();
    }
}

// One warp per sorted row: routed rows [0, offsets[e_local]) take token pair/k, shared rows
// [shared_base, shared_base + counts[e_local]) take token row - shared_base. Rows are H bf16 = H/8 uint4.
__global__ void gather_rows_kernel(const uint16_t* __restrict__ xb, const int* __restrict__ pair,
                                   const int* __restrict__ counts, const int* __restrict__ offsets, int e_local,
                                   int shared_base, int k, int H, uint16_t* __restrict__ xperm) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int routed = offsets[e_local];
    const int shared_end = shared_base + counts[e_local];
    int t;
    if (row < routed) t = pair[row] / k;
    else if (row >= shared_base && row < shared_end) t = row - shared_base;
    else return;
    const uint4* src = reinterpret_cast<const uint4*>(xb + (size_t)t * H);
    uint4* dst = reinterpret_cast<uint4*>(xperm + (size_t)row * H);
    warp_copy_row(dst, src, H / 8, lane);
}

// Work lists from a segment table seg[i] = (local expert, first row, rows) (expert parallel: the rows
// one source rank sent for one expert), plus the shared expert's rows [shared_base, +shared_rows) as
// group G = e_local. One block of 1024 threads; segments in table order.
__global__ void __launch_bounds__(1024) seg_lists_kernel(const int* __restrict__ seg, int nseg, int shared_group,
                                                         int shared_base, int shared_rows, int* __restrict__ gu_list,
                                                         int gu_bands, int gu_bands_shared, int* __restrict__ dn_list,
                                                         int dn_bands, int bn) {
    __shared__ int sh[32];
    int gu_carry = 0, dn_carry = 0;
    const int nall = nseg + (shared_rows > 0 ? 1 : 0);
    for (int i0 = 0; i0 < nall; i0 += 1024) {
        const int i = i0 + threadIdx.x;
        int g = 0, row0 = 0, cnt = 0, gub = 0;
        if (i < nseg) {
            g = seg[3 * i];
            row0 = seg[3 * i + 1];
            cnt = seg[3 * i + 2];
            gub = gu_bands;
        } else if (i < nall) {
            g = shared_group;
            row0 = shared_base;
            cnt = shared_rows;
            gub = gu_bands_shared;
        }
        const int rt = (cnt + bn - 1) / bn;
        int tgu = 0, tdn = 0;
        const int egu = block_exclusive_scan(rt * gub, sh, &tgu);
        const int edn = block_exclusive_scan(rt * dn_bands, sh, &tdn);
        if (i < nall && cnt > 0) {
            emit_tiles(gu_list, gu_carry + egu, g, gub, row0, cnt, bn);
            emit_tiles(dn_list, dn_carry + edn, g, dn_bands, row0, cnt, bn);
        }
        gu_carry += tgu;
        dn_carry += tdn;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        gu_list[0] = gu_carry;
        dn_list[0] = dn_carry;
    }
}

// Expert parallel receive side. rc[s * El + j] = rows of local expert j sent by source rank s; the rows
// arrive source-major (all of source 0's rows, local experts ascending, then source 1's, ...).
// ep_plan: seg[j] = (j, first expert-major row, rows), and per (s, j) the first source-major row
// src_off and the first expert-major row dst_off (sources ascending within an expert). One block of
// 1024 threads, El <= 1024. Counts that are negative or do not add up to R set err[1] =
// FM_EINVAL_SHAPE and leave every segment empty, so no later kernel touches a row past R.
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int* __restrict__ rc, int G, int El, int R,
                                                       int* __restrict__ seg, int* __restrict__ src_off,
                                                       int* __restrict__ dst_off, int* __restrict__ err) {
    __shared__ int sh[32];
    __shared__ int bad;
    const int j = threadIdx.x;
    if (j == 0) bad = 0;
    __syncthreads();
    int tot = 0;
    if (j < El)
        for (int s = 0; s < G; ++s) {
            const int c = rc[s * El + j];
            if (c < 0) bad = 1;
            tot += c;
        }
    int all = 0;
    const int base = block_exclusive_scan(j < El ? tot : 0, sh, &all);
    const bool ok = !bad && all == R;
    if (!ok && j == 0) atomicExch(err + 1, FM_EINVAL_SHAPE);
    if (j < El) {
        seg[3 * j] = j;
        seg[3 * j + 1] = ok ? base : 0;
        seg[3 * j + 2] = ok ? tot : 0;
        int run = base;
        for (int s = 0; s < G; ++s) {
            dst_off[s * El + j] = run;
            run += rc[s * El + j];
        }
    }
    int carry = 0;
    for (int s = 0; s < G; ++s) {
        int t = 0;
        const int ex = block_exclusive_scan(j < El ? rc[s * El + j] : 0, sh, &t);
        if (j < El) src_off[s * El + j] = carry + ex;
        carry += t;
    }
}

// One warp per expert-major row: rows [0, R) come from the received rows (the (s, j) segment holding
// source row r is the last with src_off <= r, found by binary search), rows [R, R + t_real) are this
// rank's own tokens for the shared expert. rowmap[dst] = source-major row r.
__global__ void ep_regroup_kernel(const uint16_t* __restrict__ xrecv, int R, const int* __restrict__ src_off,
                                  const int* __restrict__ dst_off, int nseg, const uint16_t* __restrict__ xb, int t_real,
                                  int H, uint16_t* __restrict__ xexp, int* __restrict__ rowmap,
                                  const int* __restrict__ err) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const uint4* src;
    int dst;
    if (row < R) {
        int lo = 0, hi = nseg - 1;   // last i with src_off[i] <= row
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (src_off[mid] <= row) lo = mid;
            else hi = mid - 1;
        }
        if (err[1]) return;   // the plan found counts that do not add up to R
        dst = dst_off[lo] + (row - src_off[lo]);
        if (dst < 0 || dst >= R) return;
        src = reinterpret_cast<const uint4*>(xrecv + (size_t)row * H);
        if (lane == 0) rowmap[dst] = row;
    } else if (row < R + t_real) {
        dst = row;
        src = reinterpret_cast<const uint4*>(xb + (size_t)(row - R) * H);
    } else {
        return;
    }
    uint4* d = reinterpret_cast<uint4*>(xexp + (size_t)dst * H);
    warp_copy_row(d, src, H / 8, lane);
}

int launch_ep_regroup(const int* rc, int G, int El, const uint16_t* xrecv, int R, const uint16_t* xb, int t_real, int H,
                      int* seg, int* src_off, int* dst_off, uint16_t* xexp, int* rowmap, int* err, cudaStream_t st) {
    ep_plan_kernel<<<1, 1024, 0, st>>>(rc, G, El, R, seg, src_off, dst_off, err);
    FM_LAUNCH_CHECK("ep_plan");
    const int rows = R + t_real;
    if (rows > 0) {
        ep_regroup_kernel<<<(rows + 7) / 8, 256, 0, st>>>(xrecv, R, src_off, dst_off, G * El, xb, t_real, H, xexp, rowmap,
                                                          err);
        FM_LAUNCH_CHECK("ep_regroup");
    }
    return FM_OK;
}

int launch_seg_lists(const int* seg, int nseg, int shared_group, int shared_base, int shared_rows, int* gu_list,
                     int gu_bands, int gu_bands_shared, int* dn_list, int dn_bands, int bn, cudaStream_t st) {
    seg_lists_kernel<<<1, 1024, 0, st>>>(seg, nseg, shared_group, shared_base, shared_rows, gu_list, gu_bands,
                                        gu_bands_shared, dn_list, dn_bands, bn);
    FM_LAUNCH_CHECK("seg_lists");
    return FM_OK;
}

int launch_dispatch(const int32_t* idx, int P, int e_begin, int e_local, int E, int shared_base, int shared_rows,
                    int* blk_hist, int nblk,
                    int* counts, int* offsets, int* pos, int* pair, int* gu_list, int gu_bands, int gu_bands_shared,
                    int* dn_list, int dn_bands, int bn, int* err, cudaStream_t st) {
    if (nblk > 0) {
        dispatch_hist_kernel<<<nblk, kDispThreads, e_local * sizeof(int), st>>>(idx, P, e_begin, e_local, E, blk_hist, err);
        FM_LAUNCH_CHECK("dispatch_hist");
    }
    dispatch_scan_kernel<<<1, 1024, 0, st>>>(blk_hist, nblk, e_local, shared_base, shared_rows, counts, offsets, gu_list, gu_bands,
                                            gu_bands_shared, dn_list, dn_bands, bn);
    FM_LAUNCH_CHECK("dispatch_scan");
    if (nblk > 0) {
        const size_t sm = (size_t)e_local * (1 + kDispThreads / 32) * sizeof(int);
        dispatch_scatter_kernel<<<nblk, kDispThreads, sm, st>>>(idx, P, e_begin, e_local, blk_hist, pos, pair);
        FM_LAUNCH_CHECK("dispatch_scatter");
    }
    return FM_OK;
}

int launch_gather(const uint16_t* xb, const int* pair, const int* counts, const int* offsets, int e_local, int shared_base,
                  int k, int H, int max_rows, uint16_t* xperm, cudaStream_t st) {
    if (max_rows <= 0) return FM_OK;
    gather_rows_kernel<<<(max_rows + 7) / 8, 256, 0, st>>>(xb, pair, counts, offsets, e_local, shared_base, k, H, xperm);
    FM_LAUNCH_CHECK("gather_rows");
    return FM_OK;
}

}  // namespace fm
