/*
 * flowmoe.h -- C ABI of libflowmoe.so, the B200 (sm_100a) Qwen3.6-MoE expert block.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t (passed as void*), returns
 * an int status (FM_OK or an FM_E* code) and never throws. fm_last_error() returns the message of the
 * calling thread's last failure. No entry point synchronises the stream unless its comment says so.
 * Threads: entry points may be called from several host threads; per-device library state (the
 * shared-expert side stream and its events) is guarded while work is enqueued. Calls on two streams of
 * one device serialise their tensor-core shared-expert work on the device's side stream. Separate
 * devices, and the decode path (T <= 128 tokens), have no such limit. No entry point calls a library
 * kernel (cuBLAS or other): every kernel launched is this library's own.
 *
 * Weights live on the device in the "tile" layout produced by fm_q4_1_to_tiles() from GGUF Q4_1
 * blocks (the reference's open_kernels/q4_1_pack.py:1-14 block format: fp16 d | fp16 m | 16 nibble
 * bytes, 32 values along K). The tile layout is a byte permutation of the same blocks (nothing is
 * re-quantised): a matrix W[N, K] (N % 128 == 0, K % 64 == 0) is cut into tiles of 128 rows x 64 K;
 * tile (band b, slab s) sits at byte ((b * K/64) + s) * 5120 and holds
 *     [0, 4096)    row r (0..127): 32 nibble bytes = the 16 nibble bytes of block 2s, then of block 2s+1,
 *                  each block's bytes b0..b15 stored as the four words [b(2c) b(2c+1) b(2c+8) b(2c+9)],
 *                  c = 0..3 (one 16x16 MMA A fragment per word, the GEMV's operand order)
 *     [4096, 5120) row r: 8 bytes = d(2s) m(2s) d(2s+1) m(2s+1), fp16
 * The down matrix [H, F] of each expert uses these 128-row bands ("down" array). Its gate and up
 * matrices [F, H] are interleaved by fm_gate_up_to_tiles() into 128-row bands of 64 features: band c
 * holds gate rows 64c..64c+63 as tile rows 0-63 and up rows 64c..64c+63 as tile rows 64-127
 * ("gate_up" array), so one tile feeds both operands of the SwiGLU.
 */
#ifndef FLOWMOE_H
#define FLOWMOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FM_API __attribute__((visibility("default")))
#else
#define FM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The reference throws std::runtime_error where these are returned. */
#define FM_OK 0
#define FM_EINVAL_SHAPE 1  /* shapes/alignment/topk > E (block_host.cpp:768) */
#define FM_EINVAL_EXPERT 2 /* an expert id out of range (core.cpp:5159-5160, :2368-2369) */
#define FM_ECUDA 3         /* a CUDA launch or runtime call failed */
#define FM_ENCCL 4         /* an NCCL call failed */
#define FM_ETIMEOUT 5      /* a bounded device wait gave up */
#define FM_EWORKSPACE 6    /* the caller's workspace is smaller than fm_workspace_size() */

/* fm_layer.flags bit: every token's expert terms are added in ascending expert order (the scatter order
 * of the reference's Core::moe_block, src/open_qwen36/core.cpp:5163-5165, :5236-5255), so a call's output is
 * bit-reproducible and independent of the other tokens in the call -- a prompt run layer by layer over
 * all its tokens gives the same bits as block by block (on one kernel path: the GEMV and the tcgen05 GEMM
 * sum a row's products in different orders). On the tcgen05 path this routes the down GEMM's y rows
 * through f32 scratch (about T * (top_k + 1) * H * 4 bytes of workspace) and a combine kernel instead of
 * atomic adds; on the GEMV path it turns off the K splits, whose count follows the call's size. */
#define FM_FIXED_ORDER 0x100

/* Activation dtypes accepted for xm. */
#define FM_F32 0
#define FM_BF16 1

/* Geometry and device weights of one MoE layer (the reference's MoeGeometry / ModelSpec MoE fields,
 * open_kernels/harness/stream_patch.hpp:33-45, recipes/spec.py:96). All pointers are device pointers
 * owned by the caller; the struct itself is read on the host only. */
typedef struct fm_layer {
    int32_t hidden;     /* H (% 128 == 0) */
    int32_t n_experts;  /* E, the router width (all experts, all ranks) */
    int32_t top_k;      /* k <= E, k <= 16 */
    int32_t ffn;        /* F, routed expert intermediate (% 64 == 0) */
    int32_t shared_ffn; /* F_s of the always-on shared expert (% 64 == 0); 0 = none */
    int32_t e_begin;    /* first expert held by this rank (expert parallel); 0 on one GPU */
    int32_t e_local;    /* experts held by this rank; E on one GPU */
    int32_t flags;      /* 0 = pick kernels by size (the GEMV up to 128 tokens while T * top_k <= 1024 and
                           e_local < 1024, else the tcgen05 grouped GEMM);
                           2 = force tcgen05, 3 = force the GEMV (within the same limits, tcgen05 past
                           them); plus FM_FIXED_ORDER; any other value is rejected (FM_EINVAL_SHAPE) */
    const uint8_t* gate_up;   /* tiles, e_local x (2 x F x H x 5/8 B): gate then up, per expert */
    const uint8_t* down;      /* tiles, e_local x (H x F x 5/8 B) */
    const uint8_t* shared_gate_up; /* tiles of the shared expert, or NULL */
    const uint8_t* shared_down;
    const uint16_t* router;   /* bf16 [E + 1, H]: router rows (Wr transposed), then the shared-gate row */
    const float* router_bias; /* f32 [E] added to the logits before the softmax, or NULL (none) */
} fm_layer;

/* Message of this thread's last failure ("" after success). Returns FM_OK. */
FM_API int fm_last_error(char* buf, size_t n);

/* Library build identity (sm arch, version). Returns FM_OK. */
FM_API int fm_version(char* buf, size_t n);

/* GGUF Q4_1 blocks uint8[rows, k/32, 20] (device) -> tile layout (device, same byte count).
 * Replaces the reference's pool packer open_kernels/q4_1_pack.py:124-142 (pack_q4_1_pool) /
 * gguf_pool/gguf_pool.py:191-213 (pack_q4_pool) for this device. rows % 128 == 0, k % 64 == 0. */
FM_API int fm_q4_1_to_tiles(const uint8_t* blocks, int32_t rows, int32_t k, uint8_t* tiles, void* stream);

/* GGUF Q4_1 gate and up blocks, each uint8[F, k/32, 20] (device) -> the interleaved gate_up tiles of
 * one expert (device, 2 x F x k x 5/8 bytes). F % 64 == 0, k % 64 == 0. */
FM_API int fm_gate_up_to_tiles(const uint8_t* gate, const uint8_t* up, int32_t F, int32_t k, uint8_t* tiles,
                               void* stream);

/* Tile layout -> GGUF Q4_1 blocks (the inverse; used to prove the repack is a permutation). */
FM_API int fm_tiles_to_q4_1(const uint8_t* tiles, int32_t rows, int32_t k, uint8_t* blocks, void* stream);

/* The reference's q4nx pool numerics (open_kernels/q4_1_pack.py:18-37, scale_dtype=bfloat16): every
 * fp16 d and m of n_tiles tiles rounded in place to bf16 precision (round to nearest even), so the
 * kernels dequantise with the narrowed scales. For bit-level agreement with the NPU's pool. */
FM_API int fm_tiles_narrow_scales(uint8_t* tiles, int64_t n_tiles, void* stream);

/* The reference's pool chunk bytes (device) -> GGUF Q4_1 blocks uint8[n, k/32, 20] (device): the
 * inverse of its pool packers, open_kernels/q4_1_pack.py:124-142 (pack_q4_1_pool: chunk_bytes 5120,
 * bf16 d and m planes) and gguf_pool/gguf_pool.py:191-213 (pack_q4_pool: chunk_bytes 6144, f32
 * planes), in the pool order of q4_1_pack.py:112-121 with band row split rs (2 standard, 4 expert
 * stripes). k % 256 == 0, n % (32 rs) == 0. Scales become fp16; *inexact (a device int32, cleared
 * here) counts those fp16 cannot hold exactly -- zero for every pool those packers write, since they
 * widen fp16 scales to f32 or narrow them to bf16. The blocks then go through fm_q4_1_to_tiles /
 * fm_gate_up_to_tiles; a 5120-byte pool's bf16 scales give the NPU pool's numerics exactly. */
FM_API int fm_pool_to_q4_1(const uint8_t* pool, int32_t n, int32_t k, int32_t rs, int32_t chunk_bytes, uint8_t* blocks,
                           int32_t* inexact, void* stream);

/* Router weight bf16 Wr [H, E] row-major (the reference's layout, block_host.cpp:775-777) and the
 * shared-expert gate bf16 sgw [H] (or NULL) -> the layer's router array bf16 [E + 1, H]. */
FM_API int fm_router_pack(const uint16_t* wr, const uint16_t* sgw, int32_t hidden, int32_t n_experts, uint16_t* router,
                   void* stream);

/* Device workspace bytes for fm_router_topk / fm_moe_block / fm_moe_layer over T tokens. */
FM_API int fm_workspace_size(const fm_layer* L, int32_t T, size_t* bytes);

/* The router over a block: logits = bf16(xm) . Wr (fp32 accumulate), softmax, top-k by probability
 * with the lowest index on a tie, renormalised; shared_gate[t] = sigmoid(bf16(xm[t]) . sgw).
 * Replaces host::router_block (src/open_qwen36/block_host.hpp:155-159, block_host.cpp:766-803).
 * xm [T, H] f32 or bf16; probs [T, E] (may be NULL); idx int32 [T, k]; w [T, k];
 * shared_gate [T] (may be NULL). */
FM_API int fm_router_topk(const fm_layer* L, const void* xm, int32_t xm_dtype, int32_t T, float* probs, int32_t* idx,
                   float* w, float* shared_gate, void* workspace, size_t workspace_bytes, void* stream);

/* The expert block: out[t] = res[t] + shared_gate[t] * shared(xm[t]) + sum over t's k experts in
 * ascending expert order of w[t,s] * down_e(bf16(silu(gate_e x) * up_e x)), x = bf16(xm[t]).
 * Rows t >= t_real are copied from res. shared_gate may be NULL (no shared expert term; the shared
 * term is also skipped when the layer has no shared expert). Expert ids outside [e_begin,
 * e_begin + e_local) are skipped on the device and counted; fm_moe_check() reports them.
 * Replaces Core::moe_block (src/open_qwen36/core.hpp:844-848, core.cpp:5150-5259) together with the
 * gated shared-expert add of Core::ffn_block (core.cpp:4342-4380). */
FM_API int fm_moe_block(const fm_layer* L, const void* xm, int32_t xm_dtype, const float* res, const int32_t* idx,
                 const float* w, const float* shared_gate, int32_t T, int32_t t_real, float* out, void* workspace,
                 size_t workspace_bytes, void* stream);

/* Router + shared expert + experts in one call (the engine's staged_tail -> ffn_block ->
 * block_layer_moe sequence, core.cpp:4934-4957 and :3685-3700). idx/w (may be NULL) receive the
 * routing. */
FM_API int fm_moe_layer(const fm_layer* L, const void* xm, int32_t xm_dtype, const float* res, int32_t T, int32_t t_real,
                 float* out, int32_t* idx, float* w, void* workspace, size_t workspace_bytes, void* stream);

/* One layer of the MoE stack: x_{l+1} = x + MoE(RMSNorm(x)). The post-attention RMSNorm (weight norm_w
 * bf16 [H], eps; Core::rmsnorm_host, core.cpp:3014-3044, fp64 reduction) is fused with the bf16
 * conversion, then the layer runs as fm_moe_layer with xm = RMSNorm(x) and res = x (the staged_tail ->
 * ffn_block sequence, core.cpp:4934-4957). x and out [T, H] f32 (out may not alias x). */
FM_API int fm_moe_layer_norm(const fm_layer* L, const float* x, const uint16_t* norm_w, float eps, int32_t T,
                             int32_t t_real, float* out, int32_t* idx, float* w, void* workspace, size_t workspace_bytes,
                             void* stream);

/* The post-attention RMSNorm alone (the first stage of fm_moe_layer_norm): xb [T, H] bf16 = bf16(x / rms(x)
 * * w), fp64 reduction, as Core::rmsnorm_host (src/open_qwen36/core.cpp:3014-3044, groups = 1). For
 * callers that feed the normalised rows to another entry point, e.g. fm_ep_peer_layer with res = x. */
FM_API int fm_rmsnorm_bf16(const float* x, const uint16_t* norm_w, float eps, int32_t T, int32_t H, uint16_t* xb,
                           void* stream);

/* Dense Q4_1 projection (the prefill projections beside the MoE block): y [T, N] f32 = bf16(x) [T, K] .
 * dequant(W) [N, K]^T, f32 accumulation, on the tcgen05 GEMM. Replaces the reference's gemm_q4_prefill
 * design (open_kernels/designs/gemm_q4_prefill/gemm_q4_prefill.py:1-3, Y[N_WEIGHT, T] = W(q4_1)[N_WEIGHT,
 * K] @ X^T[K, T]); y here is token-major, the transpose of that device layout. w_tiles = W in the tile
 * layout (fm_q4_1_to_tiles of GGUF blocks uint8[N, K/32, 20], or of fm_pool_to_q4_1's blocks for the
 * reference's pool bytes). N % 128 == 0, K % 64 == 0; x f32 or bf16 [T, K]; x, y and the workspace
 * 16-byte aligned. A device wait that gives up is reported by fm_moe_check(workspace). */
FM_API int fm_q4_gemm_workspace_size(int32_t N, int32_t K, int32_t T, int32_t x_dtype, size_t* bytes);
FM_API int fm_q4_gemm(const uint8_t* w_tiles, int32_t N, int32_t K, const void* x, int32_t x_dtype, int32_t T, float* y,
                      void* workspace, size_t workspace_bytes, void* stream);

/* The dispatch stage alone: per local expert counts [e_local], exclusive offsets [e_local + 1] (the
 * last = routed pair count), pos [t_real, k] = row of each (token, slot) pair in the expert-sorted
 * order (-1 for an id outside the local range) and pair [offsets[e_local]] = its inverse (t * k + s).
 * Within an expert, pairs keep token-then-slot order: the owed lists of core.cpp:5155-5165. Any
 * output pointer may be NULL. */
FM_API int fm_moe_dispatch(const fm_layer* L, const int32_t* idx, int32_t T, int32_t t_real, int32_t* counts,
                           int32_t* offsets, int32_t* pos, int32_t* pair, void* workspace, size_t workspace_bytes,
                           void* stream);

/* fm_moe_layer for callers that cannot allocate device memory, so it takes no workspace: an engine that
 * reserves all of its device memory when it loads a model (as the reference's engine does with fixed
 * per-layer buffers) and has no hook for a call-sized workspace, or a decode loop that cannot afford the
 * device synchronisation a cudaMalloc may cause. No counterpart in the reference.
 * The scratch space is a static 24 MiB device array in this library, held on every GPU that loads it
 * until exit; calls needing more (fm_workspace_size > 24 MiB: for 2048-wide top-8 layers more than 456
 * tokens with 128 experts of F 768, more than 497 with 256 experts of F 512 and a shared expert of 512)
 * return FM_EWORKSPACE. All calls on a device share the array, which keeps the last call's contents:
 * calls that overlap on the GPU race and must be serialised by the caller. The first call on each device
 * does a one-time set-up (it looks the array's address up and creates the side stream and events the
 * shared expert uses); make it before any stream capture. Every kernel on this path is the library's
 * own: no cudaMalloc, cudaFree or allocating library routine is called. */
FM_API int fm_moe_layer_noalloc(const fm_layer* L, const void* xm, int32_t xm_dtype, const float* res, int32_t T,
                                int32_t t_real, float* out, int32_t* idx, float* w, void* stream);

/* Expert parallel (EP) over G ranks, one process per GPU. No counterpart in the reference, which runs
 * every expert on one NPU (Core::moe_block, core.cpp:5150-5259); these three stages split that call
 * around the two all-to-all exchanges the host makes (flowmoe/ep.py, NCCL over NVLink):
 *   rank r owns experts [e_begin, e_begin + e_local) = [r * E / G, (r + 1) * E / G); the router
 *   ([E + 1, H], replicated) and the shared expert (replicated) run on each rank's own tokens.
 * Scratch needs: fm_ep_workspace_size for T own tokens and R received rows (the largest R the call
 * will see; R <= G * T * k). */
FM_API int fm_ep_workspace_size(const fm_layer* L, int32_t T, int32_t R, int32_t n_ranks, size_t* bytes);

/* Stage 1: router over all E experts (idx, w, shared_gate as fm_router_topk), then the stable
 * expert sort over ALL experts: counts [E] per expert, pos [t_real, k] = each pair's row in the sorted
 * order, and xsend [t_real * k, H] bf16 = the sorted rows. The rows for rank g are the contiguous
 * range of experts [g * e_local, (g + 1) * e_local). xb_out [T, H] receives xm as bf16 when
 * xm_dtype is FM_F32 (fm_ep_experts needs it); it may be NULL for FM_BF16 input. */
FM_API int fm_ep_dispatch(const fm_layer* L, const void* xm, int32_t xm_dtype, int32_t T, int32_t t_real,
                          uint16_t* xb_out, int32_t* idx, float* w, float* shared_gate, int32_t* counts, int32_t* pos,
                          uint16_t* xsend, void* workspace, size_t workspace_bytes, void* stream);

/* Stage 2 (after the dispatch exchange): xrecv [R, H] bf16 = the rows every rank sent here, source
 * rank major and local expert ascending within a source; recv_counts [n_ranks, e_local] (device) =
 * rows per (source, local expert). Writes out [T, H] = res + shared_gate * shared_expert(xb) for this
 * rank's own tokens (rows >= t_real: res), and yrecv [R, H] bf16 = each received row's unweighted
 * expert output, in the received order (the rows the combine exchange sends back). */
FM_API int fm_ep_experts(const fm_layer* L, const uint16_t* xrecv, int32_t R, const int32_t* recv_counts,
                         int32_t n_ranks, const uint16_t* xb, const float* shared_gate, const float* res, int32_t T,
                         int32_t t_real, float* out, uint16_t* yrecv, void* workspace, size_t workspace_bytes,
                         void* stream);

/* Stage 3 (after the combine exchange): ysorted [t_real * k, H] bf16 = the expert outputs in the
 * sorted order of stage 1; out[t] += sum of w * y over t's pairs in ascending expert order, t < t_real
 * (the weighted scatter of core.cpp:5244-5252). */
FM_API int fm_ep_combine(const fm_layer* L, float* out, const uint16_t* ysorted, const int32_t* pos, const int32_t* idx,
                         const float* w, int32_t T, int32_t t_real, void* stream);

/* ---- Expert parallel over peer memory (NVLink), no host round trip. No counterpart in the reference.
 * Every rank allocates one symmetric buffer (fm_ipc_alloc, the same size on every rank), exchanges
 * the handles (the host's all-gather) and maps its peers' buffers (fm_ipc_open). One fm_ep_peer_layer
 * call then does the whole layer: router and sort as fm_ep_dispatch; the per-expert counts stored into
 * every peer's buffer; the rows stored straight into the owning rank's receive buffer, already grouped
 * by expert; the tcgen05 expert GEMMs, whose DOWN epilogue stores each y row straight back into the
 * sending rank's buffer; the ordered weighted combine. Ranks synchronise through monotonic flags in the
 * symmetric buffers with bounded device waits: a peer that does not take its step within timeout_ms
 * makes the call end with FM_ETIMEOUT (fm_moe_check) instead of waiting for good, and no further stores
 * go to the peers. All ranks must make the same sequence of calls on one group. */
#define FM_EP_MAX_RANKS 16

typedef struct fm_ep_group {
    int32_t rank, n_ranks;           /* this process's rank, the group size (<= FM_EP_MAX_RANKS) */
    int32_t t_cap;                   /* the most tokens any rank passes to one call */
    int32_t timeout_ms;              /* bound of each device wait on the peers (0: 10000) */
    void* sym[FM_EP_MAX_RANKS];      /* each rank's symmetric buffer as mapped here; sym[rank] is our own */
} fm_ep_group;

/* Bytes of the symmetric buffer (identical on every rank) and of the per-call workspace. */
FM_API int fm_ep_peer_sizes(const fm_layer* L, const fm_ep_group* g, size_t* sym_bytes, size_t* ws_bytes);

/* The whole expert-parallel layer for this rank's T tokens (t_real real): out [T, H] f32 = res + shared
 * + routed experts, as fm_moe_layer; idx/w (may be NULL) receive the routing. */
FM_API int fm_ep_peer_layer(const fm_layer* L, const fm_ep_group* g, const void* xm, int32_t xm_dtype, const float* res,
                            int32_t T, int32_t t_real, float* out, int32_t* idx, float* w, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Device memory shareable with the other processes of the node: cudaMalloc'd, zeroed, and its
 * cudaIpcMemHandle_t (64 bytes) written to handle_out. */
FM_API int fm_ipc_alloc(size_t bytes, void** ptr, void* handle_out);
/* Maps another process's fm_ipc_alloc buffer (peer access enabled on demand). */
FM_API int fm_ipc_open(const void* handle, void** ptr);
FM_API int fm_ipc_close(void* ptr);
FM_API int fm_ipc_free(void* ptr);

/* Synchronises `stream` and returns FM_ETIMEOUT if a bounded device wait of the last call on this
 * workspace gave up, else FM_EINVAL_EXPERT if it met an expert id outside the range the block accepts
 * (the check core.cpp:5159-5160 throws on). */
FM_API int fm_moe_check(void* workspace, void* stream);

/* Launches of this library's own kernels in this process (the proof that the device path ran). */
FM_API int fm_launch_count(unsigned long long* n);

/* Stage profiler (the reference's OFLM_OPEN_PROFILE stage timings, core.cpp:592-600, :850-935, on
 * CUDA events): while enabled, each call records a timing event pair around every stage on its
 * stream. Stages: 0 to_bf16, 1 router, 2 dispatch, 3 gather, 4 gate_up, 5 down, 6 combine.
 * fm_profile(1) creates the events on first use; call it before any stream capture. Inside a captured
 * graph the records become event-record nodes, so fm_profile_read then reports the last replay. The
 * profiler is one process-wide record for one device: enable it only while a single host thread makes
 * calls (a measurement tool, not for production). */
FM_API int fm_profile(int32_t enable);

/* Waits for the recorded events and writes the summed milliseconds per stage into ms[0..n_stages),
 * then clears the record. */
FM_API int fm_profile_read(double* ms, int32_t n_stages);

#ifdef __cplusplus
}
#endif

#endif /* FLOWMOE_H */
