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
