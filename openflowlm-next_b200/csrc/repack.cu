// Weight layout kernels: GGUF Q4_1 blocks <-> the device tile layout, and the router transpose.
//
// The tile layout is a byte permutation of the GGUF blocks (open_kernels/q4_1_pack.py:1-14): nothing
// is re-quantised and the scales keep their fp16 bits. Like the reference's pool packer
// (q4_1_pack.py:124-142), it exists so the device streams one contiguous 5120-byte tile per
// (128 rows x 64 K) step instead of 20-byte blocks that straddle 16-byte boundaries.
#include "common.cuh"

namespace fm {

// Within each block's 16 nibble bytes the tile stores, for c = 0..3, the word
// [b(2c), b(2c+1), b(2c+8), b(2c+9)]: exactly the codes one mma.sync A-fragment thread needs (values
// 2c, 2c+1, 2c+8, 2c+9 in the low nibbles, +16 in the high ones), so a fragment is one 32-bit load.
__device__ __forceinline__ uint4 to_frag_order(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
    return make_uint4(__byte_perm(w0, w2, 0x5410), __byte_perm(w0, w2, 0x7632), __byte_perm(w1, w3, 0x5410),
                      __byte_perm(w1, w3, 0x7632));
}

__device__ __forceinline__ uint4 from_frag_order(uint4 t) {
    return make_uint4(__byte_perm(t.x, t.y, 0x5410), __byte_perm(t.z, t.w, 0x5410), __byte_perm(t.x, t.y, 0x7632),
                      __byte_perm(t.z, t.w, 0x7632));
}

// One thread per (row, slab): blocks 2s and 2s+1 of row r (40 bytes) -> 32 nibble bytes + 8 scale
// bytes of tile (r / 128, s). Blocks are 20 bytes = 5 words, so every block starts 4-byte aligned.
__global__ void q4_1_to_tiles_kernel(const uint32_t* __restrict__ blocks, int rows, int k, uint32_t* __restrict__ tiles) {
    const int slabs = k / kTileK;
    const long long n = (long long)rows * slabs;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / slabs), s = (int)(i % slabs);
        const uint32_t* b0 = blocks + ((long long)r * (k / 32) + 2 * s) * 5;   // block 2s
        uint32_t w[10];
#pragma unroll
        for (int j = 0; j < 10; ++j) w[j] = __ldg(b0 + j);
        const long long tile = (long long)(r / kTileRows) * slabs + s;
        const int rr = r % kTileRows;
        uint32_t* nib = tiles + tile * (kTileBytes / 4) + rr * 8;
        uint4* nib4 = reinterpret_cast<uint4*>(nib);
        nib4[0] = to_frag_order(w[1], w[2], w[3], w[4]);
        nib4[1] = to_frag_order(w[6], w[7], w[8], w[9]);
        uint2* sc = reinterpret_cast<uint2*>(tiles + tile * (kTileBytes / 4) + kTileNibBytes / 4 + rr * 2);
        *sc = make_uint2(w[0], w[5]);   // d0 m0 | d1 m1
    }
}

// gate_up layout: band c of a [F, K] pair holds gate rows 64c..64c+63 as tile rows 0-63 and up rows
// 64c..64c+63 as tile rows 64-127, so one 128-row tile feeds the SwiGLU pair of 64 features.
__global__ void gate_up_to_tiles_kernel(const uint32_t* __restrict__ gate, const uint32_t* __restrict__ up, int F, int k,
                                        uint32_t* __restrict__ tiles) {
    const int slabs = k / kTileK;
    const long long n = (long long)2 * F * slabs;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / slabs), s = (int)(i % slabs);   // r in [0, 2F): tile row order
        const int band = r / kTileRows, rr = r % kTileRows;
        const int src_row = band * 64 + (rr & 63);
        const uint32_t* b0 = (rr < 64 ? gate : up) + ((long long)src_row * (k / 32) + 2 * s) * 5;
        uint32_t w[10];
#pragma unroll
        for (int j = 0; j < 10; ++j) w[j] = __ldg(b0 + j);
        const long long tile = (long long)band * slabs + s;
        uint4* nib4 = reinterpret_cast<uint4*>(tiles + tile * (kTileBytes / 4) + rr * 8);
        nib4[0] = to_frag_order(w[1], w[2], w[3], w[4]);
        nib4[1] = to_frag_order(w[6], w[7], w[8], w[9]);
        *reinterpret_cast<uint2*>(tiles + tile * (kTileBytes / 4) + kTileNibBytes / 4 + rr * 2) = make_uint2(w[0], w[5]);
    }
}

__global__ void tiles_to_q4_1_kernel(const uint32_t* __restrict__ tiles, int rows, int k, uint32_t* __restrict__ blocks) {
    const int slabs = k / kTileK;
    const long long n = (long long)rows * slabs;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / slabs), s = (int)(i % slabs);
        const long long tile = (long long)(r / kTileRows) * slabs + s;
        const int rr = r % kTileRows;
        const uint4* nib4 = reinterpret_cast<const uint4*>(tiles + tile * (kTileBytes / 4) + rr * 8);
        const uint2 sc = *reinterpret_cast<const uint2*>(tiles + tile * (kTileBytes / 4) + kTileNibBytes / 4 + rr * 2);
        const uint4 a = from_frag_order(nib4[0]), b = from_frag_order(nib4[1]);
        uint32_t* o = blocks + ((long long)r * (k / 32) + 2 * s) * 5;
        o[0] = sc.x; o[1] = a.x; o[2] = a.y; o[3] = a.z; o[4] = a.w;
        o[5] = sc.y; o[6] = b.x; o[7] = b.y; o[8] = b.z; o[9] = b.w;
    }
}

// router[e][h] = wr[h][e] (e < E), router[E][h] = sgw[h] (or 0): one 32x32 tile per block.
__global__ void router_pack_kernel(const uint16_t* __restrict__ wr, const uint16_t* __restrict__ sgw, int H, int E,
                                   uint16_t* __restrict__ router) {
    __shared__ uint16_t t[32][33];
    const int h0 = blockIdx.x * 32, e0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int h = h0 + j, e = e0 + threadIdx.x;
        uint16_t v = 0;
        if (h < H) {
            if (e < E) v = wr[(size_t)h * E + e];
            else if (e == E && sgw) v = sgw[h];
        }
        t[j][threadIdx.x] = v;
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int e = e0 + j, h = h0 + threadIdx.x;
        if (e <= E && h < H) router[(size_t)e * H + h] = t[threadIdx.x][j];
    }
}

// The reference's pool chunk bytes -> GGUF Q4_1 blocks: the inverse of its pool packers
// (open_kernels/q4_1_pack.py:124-142 pack_q4_1_pool, 5120-byte chunks with bf16 d and m planes;
// gguf_pool/gguf_pool.py:191-213 pack_q4_pool, 6144-byte chunks with f32 planes). A chunk holds 32 rows x
// 256 K of a [n, k] matrix in the pool order of q4_1_pack.py:112-121 (chunk c: band c / per_band,
// ci = c % per_band, rows 32 rs band + 32 (ci % rs), columns 256 (ci / rs)); its scale planes are indexed
// kb * 32 + row, its codes p = (row / 16) * 4096 + col * 16 + row % 16 two to a byte, even p in the low
// nibble. One thread per (row, block): the block's d and m become fp16 (exact for every scale those
// packers write: widened fp16 values, or fp16 values narrowed to bf16); `inexact` counts the ones fp16
// cannot hold.
__global__ void pool_to_q4_1_kernel(const uint8_t* __restrict__ pool, int n, int k, int rs, int scale_bytes,
                                    uint8_t* __restrict__ blocks, int* __restrict__ inexact) {
    const int nb = k / 32;
    const long long total = (long long)n * nb;
    const int per_band = rs * k / 256;
    const int plane = 256 * scale_bytes;                  // bytes of one scale plane
    const long long chunk = 2 * plane + 4096;             // 5120 or 6144
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / nb), b = (int)(i % nb);
        const int band = r / (32 * rs), sub = (r % (32 * rs)) / 32;
        const long long c = (long long)band * per_band + (long long)(b / 8) * rs + sub;
        const uint8_t* ch = pool + c * chunk;
        const int rr = r % 32, kb = b % 8, j = kb * 32 + rr;
        float d, m;
        if (scale_bytes == 2) {
            d = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ch + 2 * j));
            m = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ch + plane + 2 * j));
        } else {
            d = *reinterpret_cast<const float*>(ch + 4 * j);
            m = *reinterpret_cast<const float*>(ch + plane + 4 * j);
        }
        const __half hd = __float2half_rn(d), hm = __float2half_rn(m);
        if (!(__half2float(hd) == d) || !(__half2float(hm) == m)) atomicAdd(inexact, 1);
        // codes of row rr, columns kb*32 .. kb*32+31 of the chunk: one nibble of every 8th byte
        const uint8_t* codes = ch + 2 * plane + ((rr >> 4) * 4096 + (rr & 15)) / 2;
        const int shift = (rr & 1) * 4;
        uint8_t q[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) q[t] = (codes[(kb * 32 + t) * 8] >> shift) & 0xF;
        uint8_t* o = blocks + i * 20;
        const unsigned short hdb = __half_as_ushort(hd), hmb = __half_as_ushort(hm);
        o[0] = hdb & 0xFF; o[1] = hdb >> 8; o[2] = hmb & 0xFF; o[3] = hmb >> 8;
#pragma unroll
        for (int t = 0; t < 16; ++t) o[4 + t] = q[t] | (q[t + 16] << 4);   // byte t: value t low, t+16 high
    }
}

}  // namespace fm

using namespace fm;

static int check_q4_geometry(int rows, int k) {
    if (rows <= 0 || k <= 0 || rows % kTileRows || k % kTileK) {
        set_error("tile layout needs rows %% 128 == 0 and k %% 64 == 0 (got rows=%d k=%d)", rows, k);
        return FM_EINVAL_SHAPE;
    }
    return FM_OK;
}

extern "C" FM_API int fm_q4_1_to_tiles(const uint8_t* blocks, int32_t rows, int32_t k, uint8_t* tiles, void* stream) {
    if (int rc = check_q4_geometry(rows, k)) return rc;
    if ((reinterpret_cast<uintptr_t>(blocks) | reinterpret_cast<uintptr_t>(tiles)) & 15) {
        set_error("fm_q4_1_to_tiles: pointers must be 16-byte aligned");
        return FM_EINVAL_SHAPE;
    }
    const long long n = (long long)rows * (k / kTileK);
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    q4_1_to_tiles_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint32_t*)blocks, rows, k, (uint32_t*)tiles);
    FM_LAUNCH_CHECK("q4_1_to_tiles");
    return FM_OK;
}

extern "C" FM_API int fm_gate_up_to_tiles(const uint8_t* gate, const uint8_t* up, int32_t F, int32_t k, uint8_t* tiles,
                                           void* stream) {
    if (F <= 0 || k <= 0 || F % 64 || k % kTileK) {
        set_error("gate_up tiles need F %% 64 == 0 and k %% 64 == 0 (got F=%d k=%d)", F, k);
        return FM_EINVAL_SHAPE;
    }
    if ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(tiles)) & 15) {
        set_error("fm_gate_up_to_tiles: pointers must be 16-byte aligned");
        return FM_EINVAL_SHAPE;
    }
    const long long n = (long long)2 * F * (k / kTileK);
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    gate_up_to_tiles_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint32_t*)gate, (const uint32_t*)up, F, k,
                                                                    (uint32_t*)tiles);
    FM_LAUNCH_CHECK("gate_up_to_tiles");
    return FM_OK;
}

extern "C" FM_API int fm_tiles_to_q4_1(const uint8_t* tiles, int32_t rows, int32_t k, uint8_t* blocks, void* stream) {
    if (int rc = check_q4_geometry(rows, k)) return rc;
    const long long n = (long long)rows * (k / kTileK);
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    tiles_to_q4_1_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint32_t*)tiles, rows, k, (uint32_t*)blocks);
    FM_LAUNCH_CHECK("tiles_to_q4_1");
    return FM_OK;
}

// q4nx numerics: every d and m of a tile array rounded to bf16 precision (round to nearest even) and
// stored back as fp16. A bf16-rounded fp16 value keeps at most 8 significant bits and its fp16
// exponent range, so the fp16 store is exact (up to an overflow at the very top of the fp16 range,
// past 65504, which Q4_1 weight scales do not reach); the kernels then see the narrowed scales.
__global__ void narrow_scales_kernel(uint8_t* __restrict__ tiles, long long n_tiles) {
    const long long n = n_tiles * (kTileBytes - kTileNibBytes) / 2;   // fp16 scale values
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long tile = i / 512, j = i % 512;
        __half* h = reinterpret_cast<__half*>(tiles + tile * kTileBytes + kTileNibBytes) + j;
        const float f = __half2float(*h);
        *h = __float2half_rn(__bfloat162float(__float2bfloat16_rn(f)));
    }
}

extern "C" FM_API int fm_tiles_narrow_scales(uint8_t* tiles, int64_t n_tiles, void* stream) {
    if (!tiles || n_tiles < 0) {
        set_error("fm_tiles_narrow_scales: null tiles or negative count");
        return FM_EINVAL_SHAPE;
    }
    if (n_tiles == 0) return FM_OK;
    const long long n = n_tiles * 512;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    narrow_scales_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(tiles, n_tiles);
    FM_LAUNCH_CHECK("narrow_scales");
    return FM_OK;
}

extern "C" FM_API int fm_pool_to_q4_1(const uint8_t* pool, int32_t n, int32_t k, int32_t rs, int32_t chunk_bytes,
                                       uint8_t* blocks, int32_t* inexact, void* stream) {
    if (!pool || !blocks || !inexact || n <= 0 || k <= 0 || rs <= 0 || k % 256 || n % (32 * rs) ||
        (chunk_bytes != 5120 && chunk_bytes != 6144)) {
        set_error("fm_pool_to_q4_1: needs k %% 256 == 0, n %% (32 rs) == 0 and 5120- or 6144-byte chunks "
                  "(got n=%d k=%d rs=%d chunk=%d)", n, k, rs, chunk_bytes);
        return FM_EINVAL_SHAPE;
    }
    if ((reinterpret_cast<uintptr_t>(pool) & 3) || (reinterpret_cast<uintptr_t>(inexact) & 3)) {
        set_error("fm_pool_to_q4_1: pool and inexact must be 4-byte aligned");
        return FM_EINVAL_SHAPE;
    }
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemsetAsync(inexact, 0, sizeof(int32_t), st) != cudaSuccess) return cuda_status(cudaGetLastError(), "memset");
    const long long total = (long long)n * (k / 32);
    const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    pool_to_q4_1_kernel<<<grid, 256, 0, st>>>(pool, n, k, rs, chunk_bytes == 5120 ? 2 : 4, blocks, inexact);
    FM_LAUNCH_CHECK("pool_to_q4_1");
    return FM_OK;
}

extern "C" FM_API int fm_router_pack(const uint16_t* wr, const uint16_t* sgw, int32_t hidden, int32_t n_experts,
                              uint16_t* router, void* stream) {
    if (hidden <= 0 || n_experts <= 0) {
        set_error("fm_router_pack: bad shape H=%d E=%d", hidden, n_experts);
        return FM_EINVAL_SHAPE;
    }
    dim3 grid((hidden + 31) / 32, (n_experts + 1 + 31) / 32);
    router_pack_kernel<<<grid, dim3(32, 8), 0, (cudaStream_t)stream>>>(wr, sgw, hidden, n_experts, router);
    FM_LAUNCH_CHECK("router_pack");
    return FM_OK;
}
