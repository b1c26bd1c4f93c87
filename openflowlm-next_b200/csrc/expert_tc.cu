// Grouped Q4_1 expert GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// One persistent CTA per SM walks the work list (group, band, first sorted row, rows). A work item
// is D[128 weight rows x n tokens] = W_band[128 x K] . X[n x K]^T with n <= 256, K walked in 64-wide
// slabs. Warp roles (448 threads):
//   warp 0      producer: per slab, one 5120-byte bulk copy of the raw Q4_1 weight tile and
//               ceil(n/32) TMA loads (128-byte swizzle) of the sorted bf16 activation rows;
//   warp 1      TMEM owner and MMA issuer: four tcgen05.mma (M=128, N=n rounded to 16, K=16) per
//               slab into one of two TMEM accumulators (2 x 256 columns), commits release the rings;
//   warps 2-5   dequantisers: thread r turns row r of the raw tile (two GGUF blocks) into 64 bf16
//               values in the 128-byte-swizzled K-major layout the MMA reads (w = q*d + m in f32 with
//               the fp16 d, m widened exactly, rounded once to bf16);
//   warps 6-13  epilogue in two halves of four warps (alternate 32-token chunks), overlapped with the
//               next item's main loop through the second accumulator:
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

constexpr int TC_EPI_WARPS = 8;
constexpr int TC_THREADS = 32 * (6 + TC_EPI_WARPS);   // producer, MMA, 4 dequantisers, 8 epilogue warps
constexpr int TC_BN = 256;                 // max tokens per work item (MMA N)
constexpr int TC_SR = 4;                   // raw weight tile ring
constexpr int TC_SB = 4;                   // activation tile ring
constexpr int TC_SA = 2;                   // dequantised A tile ring
constexpr int TC_A_BYTES = 128 * 128;      // 128 rows x 64 bf16
constexpr int TC_B_BYTES = TC_BN * 128;    // 256 rows x 64 bf16
constexpr int TC_BOX_ROWS = 32;
constexpr int TC_EPI_LD = 132;             // padded f32 row of the DOWN staging tile
// epilogue staging: GATE_UP gate/up exchange (2 x 16 x 64 f32) + h tile (32 x 64 bf16);
// DOWN weighted y tile (32 x 132 f32) + token / weight lists (2 x 256)
constexpr int TC_HALF_BYTES = 32 * TC_EPI_LD * 4;            // one epilogue half's staging area
constexpr int TC_EPI_BYTES = 2 * TC_HALF_BYTES + 2 * 256 * 4;   // two halves + token / weight lists

struct TcSmem {
    // offsets from the 1024-aligned dynamic smem base
    static constexpr int a = 0;
    static constexpr int b = a + TC_SA * TC_A_BYTES;
    static constexpr int raw = b + TC_SB * TC_B_BYTES;
    static constexpr int epi = raw + TC_SR * kTileBytes;
    static constexpr int bars = epi + TC_EPI_BYTES;
    static constexpr int nbars = 2 * TC_SR + 2 * TC_SB + 2 * TC_SA + 4;
    static constexpr int tmem = bars + nbars * 8;
    static constexpr int total = tmem + 16 + 1024;   // + alignment slack
};

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

template <bool GATE_UP>
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
__global__ void __launch_bounds__(TC_THREADS, 1) expert_tc_kernel(const __grid_constant__ CUtensorMap bmap, TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcSmem::bars);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = raw_full + TC_SR;
    uint64_t* b_full = raw_empty + TC_SR;
    uint64_t* b_empty = b_full + TC_SB;
    uint64_t* a_full = b_empty + TC_SB;
    uint64_t* a_empty = a_full + TC_SA;
    uint64_t* acc_full = a_empty + TC_SA;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TcSmem::tmem);
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = a.list[0];

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int i = 0; i < TC_SR; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], 128); }
        for (int i = 0; i < TC_SB; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
        for (int i = 0; i < TC_SA; ++i) { mbar_init(&a_full[i], 128); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 32 * TC_EPI_WARPS); }
        mbar_fence_init();
        prefetch_tmap(&bmap);
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
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int rs = 0, bs = 0;
            uint32_t rph = 0, bph = 0;
            uint32_t issued_r = 0, issued_b = 0;   // bit i: slot i has a fill in flight or landed
            bool ok = true;
            for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
                const Item it = decode_item<GATE_UP>(a, i);
                const int nb = (it.n + TC_BOX_ROWS - 1) / TC_BOX_ROWS;
                for (int s = 0; s < it.slabs; ++s) {
                    if (!mbar_wait(&raw_empty[rs], rph ^ 1)) { ok = false; break; }
                    mbar_expect_tx(&raw_full[rs], kTileBytes);
                    bulk_load(smem + TcSmem::raw + rs * kTileBytes, it.w + (size_t)s * kTileBytes, kTileBytes, &raw_full[rs]);
                    issued_r |= 1u << rs;
                    if (!mbar_wait(&b_empty[bs], bph ^ 1)) { ok = false; break; }
                    mbar_expect_tx(&b_full[bs], nb * TC_BOX_ROWS * 128);
                    for (int j = 0; j < nb; ++j)
                        tma_load_2d(smem + TcSmem::b + bs * TC_B_BYTES + j * TC_BOX_ROWS * 128, &bmap, s * kTileK,
                                    it.row0 + j * TC_BOX_ROWS, &b_full[bs]);
                    issued_b |= 1u << bs;
                    if (++rs == TC_SR) { rs = 0; rph ^= 1; }
                    if (++bs == TC_SB) { bs = 0; bph ^= 1; }
                }
            }
            if (!ok) {
                fail(a.err, FM_ETIMEOUT);
                atomicExch(&abort_flag, 1);
                // drain: every slot's most recent fill must land before the CTA may exit
                for (int i = 0; i < TC_SR; ++i) {
                    const int slot = (rs + i) % TC_SR;
                    const uint32_t ph = slot < rs ? rph : rph ^ 1;   // parity of the slot's last fill
                    if (issued_r >> slot & 1u) mbar_wait(&raw_full[slot], ph);
                }
                for (int i = 0; i < TC_SB; ++i) {
                    const int slot = (bs + i) % TC_SB;
                    const uint32_t ph = slot < bs ? bph : bph ^ 1;
                    if (issued_b >> slot & 1u) mbar_wait(&b_full[slot], ph);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int as = 0, bs = 0;
            uint32_t aph = 0, bph = 0;
            bool ok = true;
            int local = 0;
            for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++local) {
                const Item it = decode_item<GATE_UP>(a, i);
                const int acc = local & 1;
                const uint32_t accph = (local >> 1) & 1;
                if (!mbar_wait(&acc_empty[acc], accph ^ 1)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * 256;
                const int N = (it.n + 15) & ~15;
                const uint32_t idesc = idesc_bf16(128, N);
                for (int s = 0; s < it.slabs; ++s) {
                    if (!mbar_wait(&a_full[as], aph) || !mbar_wait(&b_full[bs], bph)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + TcSmem::a + as * TC_A_BYTES);
                    const uint32_t sb = smem_u32(smem + TcSmem::b + bs * TC_B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_f16(d_tmem, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + kk * 32), idesc,
                                   (s > 0 || kk > 0) ? 1u : 0u);
                    tc_commit(&a_empty[as]);
                    tc_commit(&b_empty[bs]);
                    if (++as == TC_SA) { as = 0; aph ^= 1; }
                    if (++bs == TC_SB) { bs = 0; bph ^= 1; }
                }
                if (!ok) break;
                tc_commit(&acc_full[acc]);
            }
            if (!ok) {
                fail(a.err, FM_ETIMEOUT);
                atomicExch(&abort_flag, 1);
            }
        }
    } else if (warp < 6) {
        // ------------------------------------------------------------ dequantisers
        const int r = threadIdx.x - 64;   // row of the 128-row tile
        int rs = 0, as = 0;
        uint32_t rph = 0, aph = 0;
        bool ok = true;
        for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
            const Item it = decode_item<GATE_UP>(a, i);
            for (int s = 0; s < it.slabs; ++s) {
                if (!mbar_wait(&raw_full[rs], rph)) { ok = false; break; }
                const uint8_t* raw = smem + TcSmem::raw + rs * kTileBytes;
                const uint4 n0 = gguf_order(*reinterpret_cast<const uint4*>(raw + r * 32));
                const uint4 n1 = gguf_order(*reinterpret_cast<const uint4*>(raw + r * 32 + 16));
                const uint2 sc = *reinterpret_cast<const uint2*>(raw + kTileNibBytes + r * 8);
                mbar_arrive(&raw_empty[rs]);
                const float d0 = __half2float(__ushort_as_half((unsigned short)(sc.x & 0xFFFF)));
                const float m0 = __half2float(__ushort_as_half((unsigned short)(sc.x >> 16)));
                const float d1 = __half2float(__ushort_as_half((unsigned short)(sc.y & 0xFFFF)));
                const float m1 = __half2float(__ushort_as_half((unsigned short)(sc.y >> 16)));
                uint4 ch[8];
                deq_block(n0, d0, m0, ch);
                deq_block(n1, d1, m1, ch + 4);
                if (!mbar_wait(&a_empty[as], aph ^ 1)) { ok = false; break; }
                uint8_t* arow = smem + TcSmem::a + as * TC_A_BYTES + r * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) = ch[c];
                fence_proxy_async_smem();
                mbar_arrive(&a_full[as]);
                if (++rs == TC_SR) { rs = 0; rph ^= 1; }
                if (++as == TC_SA) { as = 0; aph ^= 1; }
            }
        }
        if (!ok) {
            fail(a.err, FM_ETIMEOUT);
            atomicExch(&abort_flag, 1);
        }
    } else {
        // ------------------------------------------------------------ epilogue (8 warps, 2 halves)
        // Warp w reads TMEM lane group w % 4; the half (w - 6) / 4 takes every other 32-column chunk
        // (c0 = 32 half + 64 i) with its own staging area and named barrier (1 + half, 128 threads);
        // barrier 3 spans all 256 epilogue threads.
        const int lg = warp & 3;                 // TMEM lane group this warp may access
        const int row = lg * 32 + lane;          // accumulator row = TMEM lane
        const int et = threadIdx.x - 192;        // 0..255
        const int half = et >> 7;
        const int ht = et & 127;                 // thread within the half
        const int hbar = 1 + half;
        uint8_t* epi = smem + TcSmem::epi + half * TC_HALF_BYTES;
        float* xg = reinterpret_cast<float*>(epi);                   // GATE_UP: gate, cols 16-31 [16][64]
        float* xu = xg + 16 * 64;                                    //          up, cols 0-15 [16][64]
        uint16_t* hst = reinterpret_cast<uint16_t*>(xu + 16 * 64);   //          h tile [32][64] bf16
        float* ys = reinterpret_cast<float*>(epi);                   // DOWN: weighted y [32][TC_EPI_LD]
        int* tok = reinterpret_cast<int*>(smem + TcSmem::epi + 2 * TC_HALF_BYTES);   // token per row [256]
        float* wgt = reinterpret_cast<float*>(tok + 256);                            // weight per row [256]
        __shared__ int epi_abort;
        if (et == 0) epi_abort = 0;
        named_bar(3, 256);
        int local = 0;
        for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++local) {
            const Item it = decode_item<GATE_UP>(a, i);
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
            named_bar(3, 256);
            if (epi_abort) break;
            if (!GATE_UP) {
                if (et < it.n) {
                    tok[et] = tk;
                    wgt[et] = wk;
                }
                named_bar(3, 256);
            }
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(lg * 32) << 16) + acc * 256;
            for (int c0 = 32 * half; c0 < it.n; c0 += 64) {
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
            mbar_arrive(&acc_empty[acc]);
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

// bf16 matrix [rows, cols] with row stride ld elements -> map with a {64, 32} box, 128-byte swizzle.
static int make_bmap(CUtensorMap* m, const uint16_t* base, int rows, int cols, int ld) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return FM_ECUDA;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {64, TC_BOX_ROWS};
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

static int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

int launch_expert_tc(bool gate_up, const TcLaunch& L, cudaStream_t st) {
    if (L.max_items <= 0) return FM_OK;
    CUtensorMap bmap;
    if (int rc = make_bmap(&bmap, L.act, L.act_rows, L.act_cols, L.act_ld)) return rc;
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
    const int grid = L.max_items < sm_count() ? L.max_items : sm_count();
    const int sm = TcSmem::total;
    if (gate_up) {
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(expert_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
            attr = true;
        }
        expert_tc_kernel<true><<<grid, TC_THREADS, sm, st>>>(bmap, a);
    } else {
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(expert_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
            attr = true;
        }
        expert_tc_kernel<false><<<grid, TC_THREADS, sm, st>>>(bmap, a);
    }
    FM_LAUNCH_CHECK(gate_up ? "expert_tc<gate_up>" : "expert_tc<down>");
    return FM_OK;
}

}  // namespace fm
