// Shared device helpers of libflowmoe (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "flowmoe.h"

namespace fm {

constexpr int kTileRows = 128;       // rows of a weight tile (one tcgen05 M=128 band)
constexpr int kTileK = 64;           // K of a weight tile (two Q4_1 blocks, one 128 B bf16 row)
constexpr int kTileBytes = 5120;     // 128 rows x (32 nibble bytes + 8 scale bytes)
constexpr int kTileNibBytes = 4096;  // nibble area of a tile
constexpr int kMaxTopK = 16;
constexpr int kMaxRanks = FM_EP_MAX_RANKS;   // expert-parallel group size limit

// Status recorded by the host API for the calling thread.
void set_error(const char* fmt, ...);
void clear_error();   // an entry point's first step: the calling thread's message is for this call only
int cuda_status(cudaError_t e, const char* what);

// Kernel launches made by this library in this process (reported by fm_launch_count).
void note_launch();

// SMs of the current device (cached per device).
int device_sm_count();

// Raises a kernel's dynamic shared-memory limit on the current device to at least `bytes` (never
// lowers it): the attribute is per device; a mutex makes concurrent first calls safe.
cudaError_t raise_smem_limit(const void* func, int bytes);

// Launch-error check after each kernel launch: counts the launch, returns FM_ECUDA with the message
// of the last launch error.
#define FM_LAUNCH_CHECK(what)                                        \
    do {                                                             \
        ::fm::note_launch();                                         \
        cudaError_t e_ = cudaGetLastError();                         \
        if (e_ != cudaSuccess) return ::fm::cuda_status(e_, what);   \
    } while (0)

// Programmatic dependent launch on the decode-size chain (RMSNorm / bf16 conversion, router, single-CTA
// dispatch, GEMVs, combine): each of those kernels may be scheduled while the one before it in the
// stream still runs, so its launch latency and prologue overlap that kernel. On unless the environment
// sets FLOWMOE_PDL=0.
bool pdl_on();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_on() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Launch through launch_pdl, counted and checked like FM_LAUNCH_CHECK.
#define FM_LAUNCH_PDL(what, kern, grid, block, smem, st, ...)                                \
    do {                                                                                     \
        ::fm::note_launch();                                                                 \
        cudaError_t e_ = ::fm::launch_pdl(kern, grid, block, smem, st, __VA_ARGS__);         \
        const cudaError_t l_ = cudaGetLastError();                                           \
        if (e_ == cudaSuccess) e_ = l_;                                                      \
        if (e_ != cudaSuccess) return ::fm::cuda_status(e_, what);                           \
    } while (0)

// The device side of a programmatically launched kernel. pdl_wait() returns once the kernel before it
// in the stream has completed and its writes are visible (at once for an ordinary launch); such a
// kernel calls it before its first access to memory that earlier work writes or reads. Because every
// kernel of the chain waits so, each one completes only after all work before it. pdl_launch_dependents()
// lets the next kernel's CTAs be scheduled; it is called after pdl_wait(), so a kernel that starts early
// finds everything two launches back complete.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Stage timing (fm_profile): CUDA events around each stage on the launching stream.
enum Stage { kStageToBf16 = 0, kStageRouter, kStageDispatch, kStageGather, kStageGateUp, kStageDown, kStageCombine,
             kStageCount };
void prof_begin(int stage, cudaStream_t st);
void prof_end(int stage, cudaStream_t st);

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// f32 -> bf16 bits, round to nearest even (the reference's f32_to_bf16 / replica_block.bf16_round;
// NaN is not produced by the block's arithmetic on finite inputs).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide exclusive scan of one int per thread (blockDim.x == 1024). Returns the total in *total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* sh, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int s = sh[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        sh[lane] = s;   // inclusive warp totals
    }
    __syncthreads();
    const int base = warp ? sh[warp - 1] : 0;
    const int t = sh[31];
    __syncthreads();
    if (total) *total = t;
    return base + x - v;
}

// One warp copies a row of n16 16-byte words: each lane issues up to 8 loads before its stores, so a
// row's loads are in flight together.
__device__ __forceinline__ void warp_copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int n16, int lane) {
    for (int c0 = lane; c0 < n16; c0 += 32 * 8) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (c0 + 32 * u < n16) v[u] = __ldg(src + c0 + 32 * u);
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (c0 + 32 * u < n16) dst[c0 + 32 * u] = v[u];
    }
}

// Workspace layout shared by the entry points (byte offsets, 256-aligned). Built on the host.
struct Workspace {
    size_t logits;      // f32 [T, E+1]
    size_t err;         // i32 [4]: [0] bad expert ids seen
    size_t counts;      // i32 [G] per group rows (G = e_local + 1, the shared expert last)
    size_t offsets;     // i32 [G + 1]
    size_t blk_hist;    // i32 [nblk, e_local]
    size_t pos;         // i32 [T * k]: sorted row of each (token, slot) pair, -1 when skipped
    size_t pair;        // i32 [T * k]: sorted row -> pair id
    size_t tiles;       // i32 [max_tiles * 4]: (group, band, row0, nrows) work list + header
    size_t xperm;       // bf16 [T * k, H] gathered activations, sorted by expert
    size_t hperm;       // bf16 [T * k + T, F_max] SwiGLU outputs, sorted rows then the shared rows
    size_t yperm;       // f32 [T * k + T, H] down outputs, same rows as hperm
    size_t sgate;       // f32 [T] shared gate
    size_t total;
    int nblk;
    int max_tiles;
};

}  // namespace fm
